// Table-driven Muon kernels: one launch for work that the optimizer would otherwise issue once per matrix unit.
//
// Role of the reference's Muon-add lever (baselines/PixelGen/src/optim/muon_add.py:9-35: `W += alpha_k O_k` for every
// unit from a device pointer table, one Triton launch) and of the per-unit Nesterov inputs stacked for the batched
// Newton-Schulz (baselines/PixelGen/src/optim/muon.py:150-216). A d12 model has 219 units (q, k, v, k_y, v_y, proj, the
// two SwiGLU halves, w3 and the six adaLN parts of every block); issued one by one, their lerps, copies and adds are
// ~660 tiny launches per step that leave the GPU waiting on the host.
//
// muon_gather: rows [dst*, grad fp32*, momentum fp32*, numel]: optionally momentum = lerp(momentum, grad, 1 - beta)
//              first (written back), then dst = nesterov ? lerp(grad, momentum, beta) : momentum, with torch.lerp's
//              formula (the end-anchored form for weights >= 0.5); dst fp32 or bf16.
// muon_apply:  rows [param fp32*, update bf16*, numel, coef (fp32 bits)(, ema fp32*)]: param = param * decay + coef *
//              update (then the EMA's lerp toward it when the row has an EMA buffer).
// numel is a multiple of 4 and every pointer is 16-byte aligned (row slices of contiguous matrices); the host checks.
#include <ATen/cuda/CUDAContext.h>
#include <cmath>
#include <vector>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include "status.h"

namespace ng {

__device__ __forceinline__ float lerp_torch(float a, float b, float w) {
  return fabsf(w) < 0.5f ? a + w * (b - a) : b - (b - a) * (1.0f - w);
}

// mom >= 0: the momentum update m = lerp(m, grad, mom) (torch._foreach_lerp_'s formula) happens in the same pass and
// m is written back; out_bf16: dst holds bf16 (the Newton-Schulz input's precision: the same rounding as a later
// .to(bfloat16)).
__global__ void muon_gather_kernel(const int64_t* __restrict__ tab, float beta, int nesterov, float mom,
                                   int out_bf16) {
  const int64_t* r = tab + (int64_t)blockIdx.y * 4;
  const float4* g = reinterpret_cast<const float4*>(r[1]);
  float4* m = reinterpret_cast<float4*>(r[2]);
  const int64_t n4 = r[3] / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 mv = m[i];
    const float4 gv = (nesterov || mom >= 0.f) ? g[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (mom >= 0.f) {
      mv = make_float4(lerp_torch(mv.x, gv.x, mom), lerp_torch(mv.y, gv.y, mom), lerp_torch(mv.z, gv.z, mom),
                       lerp_torch(mv.w, gv.w, mom));
      m[i] = mv;
    }
    const float4 o = nesterov ? make_float4(lerp_torch(gv.x, mv.x, beta), lerp_torch(gv.y, mv.y, beta),
                                            lerp_torch(gv.z, mv.z, beta), lerp_torch(gv.w, mv.w, beta))
                              : mv;
    if (out_bf16) {
      uint2 pk;
      pk.x = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(o.x)) |
             ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(o.y)) << 16);
      pk.y = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(o.z)) |
             ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(o.w)) << 16);
      reinterpret_cast<uint2*>(r[0])[i] = pk;
    } else {
      reinterpret_cast<float4*>(r[0])[i] = o;
    }
  }
}

// rows [param fp32*, update bf16*, numel, coef (fp32 bits), ema fp32* or 0] (width 5; the width-4 form has no EMA
// column); with an EMA buffer also ema = lerp(ema, param, ema_w) after the update
__global__ void muon_apply_kernel(const int64_t* __restrict__ tab, int width, float decay, float ema_w) {
  const int64_t* r = tab + (int64_t)blockIdx.y * width;
  float4* p = reinterpret_cast<float4*>(r[0]);
  const uint2* u = reinterpret_cast<const uint2*>(r[1]);  // 4 bf16
  const int64_t n4 = r[2] / 4;
  const float coef = __int_as_float((int)r[3]);
  float4* e = width > 4 ? reinterpret_cast<float4*>(r[4]) : nullptr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const uint2 w = u[i];
    float4 v = p[i];
    v.x = v.x * decay + coef * __uint_as_float(w.x << 16);
    v.y = v.y * decay + coef * __uint_as_float(w.x & 0xFFFF0000u);
    v.z = v.z * decay + coef * __uint_as_float(w.y << 16);
    v.w = v.w * decay + coef * __uint_as_float(w.y & 0xFFFF0000u);
    p[i] = v;
    if (e != nullptr) {
      float4 ev = e[i];
      ev.x = lerp_torch(ev.x, v.x, ema_w);
      ev.y = lerp_torch(ev.y, v.y, ema_w);
      ev.z = lerp_torch(ev.z, v.z, ema_w);
      ev.w = lerp_torch(ev.w, v.w, ema_w);
      e[i] = ev;
    }
  }
}

// adamw_apply: rows [param fp32*, grad fp32*, exp_avg fp32*, exp_avg_sq fp32*, ema fp32* or 0, numel] and this
// step's scalars: the AdamW update of every row in one launch (decoupled weight decay, torch.optim.AdamW's formula:
// p *= 1 - lr wd; m = lerp(m, g, 1 - b1); v = b2 v + (1 - b2) g^2; p -= (lr / bc1) m / (sqrt(v) / sqrt(bc2) + eps)),
// then, for rows with an EMA buffer, ema = lerp(ema, p, 1 - decay). Role of the reference's FusedAdamWEMA lever
// (baselines/PixelGen/src/utils/fused_adamw_ema.py:39-113: clip, AdamW and EMA from one pointer table); gradients
// arrive already clipped here (the trainer scales them by the clip coefficient once for all parameters).
struct AdamScalars {
  float lr, wd, b1, b2, eps, step_size, rsqrt_bc2, ema_w;  // step_size = lr / bc1, ema_w = 1 - decay
};

__global__ void adamw_apply_kernel(const int64_t* __restrict__ tab, AdamScalars sc) {
  const int64_t* r = tab + (int64_t)blockIdx.y * 6;
  float4* p = reinterpret_cast<float4*>(r[0]);
  const float4* g = reinterpret_cast<const float4*>(r[1]);
  float4* m = reinterpret_cast<float4*>(r[2]);
  float4* v = reinterpret_cast<float4*>(r[3]);
  float4* e = reinterpret_cast<float4*>(r[4]);
  const int64_t n4 = r[5] / 4;
  const float keep = 1.f - sc.lr * sc.wd;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float pa[4], ga[4], ma[4], va[4];
    *reinterpret_cast<float4*>(pa) = p[i];
    *reinterpret_cast<float4*>(ga) = g[i];
    *reinterpret_cast<float4*>(ma) = m[i];
    *reinterpret_cast<float4*>(va) = v[i];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      ma[k] = lerp_torch(ma[k], ga[k], 1.f - sc.b1);
      va[k] = sc.b2 * va[k] + (1.f - sc.b2) * ga[k] * ga[k];
      const float denom = sqrtf(va[k]) * sc.rsqrt_bc2 + sc.eps;
      pa[k] = pa[k] * keep - sc.step_size * (ma[k] / denom);
    }
    p[i] = *reinterpret_cast<float4*>(pa);
    m[i] = *reinterpret_cast<float4*>(ma);
    v[i] = *reinterpret_cast<float4*>(va);
    if (e != nullptr) {
      float ea[4];
      *reinterpret_cast<float4*>(ea) = e[i];
#pragma unroll
      for (int k = 0; k < 4; ++k) ea[k] = lerp_torch(ea[k], pa[k], sc.ema_w);
      e[i] = *reinterpret_cast<float4*>(ea);
    }
  }
}

static dim3 table_grid(const at::Tensor& tab, int64_t max_numel, int64_t width = 4) {
  TORCH_CHECK(tab.is_cuda() && tab.scalar_type() == at::kLong && tab.dim() == 2 && tab.size(1) == width &&
                  tab.is_contiguous(),
              "optimizer table: [rows, width] int64 CUDA tensor expected");
  TORCH_CHECK(tab.size(0) <= 65535, "muon table: at most 65535 rows");
  const int64_t blocks = std::min<int64_t>((max_numel / 4 + 255) / 256, 64);
  return dim3((unsigned)std::max<int64_t>(blocks, 1), (unsigned)tab.size(0));
}

void muon_gather(const at::Tensor& tab, double beta, bool nesterov, int64_t max_numel, double mom, bool out_bf16) {
  if (tab.size(0) == 0) return;
  const at::cuda::CUDAGuard guard(tab.device());
  muon_gather_kernel<<<table_grid(tab, max_numel), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      tab.data_ptr<int64_t>(), (float)beta, nesterov ? 1 : 0, (float)mom, out_bf16 ? 1 : 0);
  NG_LAUNCH_CHECK();
}

void muon_apply(const at::Tensor& tab, double decay, int64_t max_numel, double ema_w) {
  if (tab.size(0) == 0) return;
  const at::cuda::CUDAGuard guard(tab.device());
  const int64_t width = tab.dim() == 2 ? tab.size(1) : 0;
  TORCH_CHECK(width == 4 || width == 5, "muon_apply: table rows of 4 (no EMA) or 5 columns");
  muon_apply_kernel<<<table_grid(tab, max_numel, width), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      tab.data_ptr<int64_t>(), (int)width, (float)decay, (float)ema_w);
  NG_LAUNCH_CHECK();
}

// scalars: lr, wd, b1, b2, eps, bias correction 1, bias correction 2, EMA weight (1 - decay; ignored for rows
// without an EMA buffer)
void adamw_apply(const at::Tensor& tab, std::vector<double> scalars, int64_t max_numel) {
  if (tab.size(0) == 0) return;
  TORCH_CHECK(scalars.size() == 8, "adamw_apply: 8 scalars");
  const at::cuda::CUDAGuard guard(tab.device());
  AdamScalars sc;
  sc.lr = (float)scalars[0];
  sc.wd = (float)scalars[1];
  sc.b1 = (float)scalars[2];
  sc.b2 = (float)scalars[3];
  sc.eps = (float)scalars[4];
  sc.step_size = (float)(scalars[0] / scalars[5]);
  sc.rsqrt_bc2 = (float)(1.0 / std::sqrt(scalars[6]));
  sc.ema_w = (float)scalars[7];
  adamw_apply_kernel<<<table_grid(tab, max_numel, 6), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      tab.data_ptr<int64_t>(), sc);
  NG_LAUNCH_CHECK();
}

}  // namespace ng
