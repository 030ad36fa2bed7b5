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
#include <algorithm>
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

// ------------------------------------------------------------------------------------------- clip and Newton-Schulz
// scale_by: buf *= *coef (the clip coefficient, read on the device: no host sync), float4 vectors; n % 4 == 0.
__global__ void scale_by_kernel(float4* __restrict__ buf, int64_t n4, const float* __restrict__ coef) {
  const float c = *coef;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = buf[i];
    v.x *= c;
    v.y *= c;
    v.z *= c;
    v.w *= c;
    buf[i] = v;
  }
}

void scale_by(const at::Tensor& buf, const at::Tensor& coef) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kFloat && buf.is_contiguous() && buf.numel() % 4 == 0 &&
                  (reinterpret_cast<uintptr_t>(buf.data_ptr()) & 15) == 0,
              "scale_by: contiguous, 16-byte aligned fp32 buffer of a multiple of 4 values");
  TORCH_CHECK(coef.is_cuda() && coef.scalar_type() == at::kFloat && coef.numel() == 1, "scale_by: one fp32 coef");
  const int64_t n4 = buf.numel() / 4;
  if (n4 == 0) return;
  const at::cuda::CUDAGuard guard(buf.device());
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, buf.get_device());
  const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, 8 * (int64_t)sms);
  scale_by_kernel<<<(unsigned)blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<float4*>(buf.data_ptr()), n4, coef.data_ptr<float>());
  NG_LAUNCH_CHECK();
}

// Newton-Schulz input: per matrix of a batch [n, a, b] bf16, X / (||X||_F + 1e-7) as PyTorch evaluates it on bf16
// tensors (the norm rounded to bf16, then + 1e-7 in bf16, then an IEEE division rounded to bf16), optionally written
// transposed ([n, b, a]: tall matrices iterate on X^T). Two kernels: per-CTA sums of squares of row chunks, then the
// scale (+ transpose) pass, in which one warp of every CTA adds its matrix's partials in a fixed order (deterministic).
constexpr int NS_ROWS = 16;  // rows per CTA of the sum-of-squares pass

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__global__ void ns_sumsq_kernel(const __nv_bfloat16* __restrict__ x, int a, int b, float* __restrict__ part) {
  __shared__ float red[8];
  const int item = blockIdx.y, chunk = blockIdx.x;
  const int r0 = chunk * NS_ROWS, r1 = min(a, r0 + NS_ROWS);
  const __nv_bfloat16* base = x + (int64_t)item * a * b;
  float acc = 0.f;
  const int nv = b / 8;  // 16-byte vectors per row
  for (int r = r0; r < r1; ++r)
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
      const uint4 u = reinterpret_cast<const uint4*>(base + (int64_t)r * b)[v];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float lo = __uint_as_float(w[k] << 16), hi = __uint_as_float(w[k] & 0xffff0000u);
        acc += lo * lo + hi * hi;
      }
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
    part[(int64_t)item * gridDim.x + chunk] = t;
  }
}

// The divisor of one matrix from its chunk partials, summed by one warp in a fixed order (lane-strided, then a
// butterfly): the same value in every CTA of the matrix. Call with all 32 lanes of a warp.
__device__ __forceinline__ float ns_den(const float* __restrict__ p, int chunks) {
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
  for (int k = lane; k < chunks; k += 32) ss += p[k];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return bf16_round(bf16_round(sqrtf(ss)) + 1e-7f);
}

// untransposed: 8 values per thread (16-byte vectors), a CTA per (row block, matrix)
__global__ void ns_scale_vec_kernel(const __nv_bfloat16* __restrict__ x, int64_t per_item, const float* __restrict__ part,
                                    int chunks, __nv_bfloat16* __restrict__ out) {
  __shared__ float s_den;
  const int item = blockIdx.y;
  if (threadIdx.x < 32) {
    const float d = ns_den(part + (int64_t)item * chunks, chunks);
    if (threadIdx.x == 0) s_den = d;
  }
  __syncthreads();
  const float den = s_den;
  const uint4* in = reinterpret_cast<const uint4*>(x + (int64_t)item * per_item);
  uint4* o = reinterpret_cast<uint4*>(out + (int64_t)item * per_item);
  const int64_t nv = per_item / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    uint4 u = in[i];
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float lo = __fdiv_rn(__uint_as_float(w[k] << 16), den);
      const float hi = __fdiv_rn(__uint_as_float(w[k] & 0xffff0000u), den);
      w[k] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
             ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
    }
    o[i] = u;
  }
}

// transposed: 32 x 32 tiles (8 warps, 4 rows each): out[item] = in[item]^T / den[item]
__global__ void ns_scale_kernel(const __nv_bfloat16* __restrict__ x, int a, int b, const float* __restrict__ part,
                                int chunks, int transpose, __nv_bfloat16* __restrict__ out) {
  __shared__ float tile[32][33];
  __shared__ float s_den;
  const int item = blockIdx.z;
  if (threadIdx.y == 0) s_den = ns_den(part + (int64_t)item * chunks, chunks);
  __syncthreads();
  const float den = s_den;
  const __nv_bfloat16* in = x + (int64_t)item * a * b;
  __nv_bfloat16* o = out + (int64_t)item * a * b;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int r = r0 + k, c = c0 + threadIdx.x;
    float v = 0.f;
    if (r < a && c < b) v = __fdiv_rn(__bfloat162float(in[(int64_t)r * b + c]), den);
    tile[k][threadIdx.x] = v;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    if (transpose) {  // out [b, a]: row c0 + k, column r0 + x
      const int r = c0 + k, c = r0 + threadIdx.x;
      if (r < b && c < a) o[(int64_t)r * a + c] = __float2bfloat16_rn(tile[threadIdx.x][k]);
    } else {
      const int r = r0 + k, c = c0 + threadIdx.x;
      if (r < a && c < b) o[(int64_t)r * b + c] = __float2bfloat16_rn(tile[k][threadIdx.x]);
    }
  }
}

// batched transpose of bf16 matrices [n, a, b] -> [n, b, a] (the Newton-Schulz output of tall matrices)
__global__ void transpose_bf16_kernel(const __nv_bfloat16* __restrict__ x, int a, int b,
                                      __nv_bfloat16* __restrict__ out) {
  __shared__ __nv_bfloat16 tile[32][34];
  const int item = blockIdx.z;
  const __nv_bfloat16* in = x + (int64_t)item * a * b;
  __nv_bfloat16* o = out + (int64_t)item * a * b;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int r = r0 + k, c = c0 + threadIdx.x;
    if (r < a && c < b) tile[k][threadIdx.x] = in[(int64_t)r * b + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int r = c0 + k, c = r0 + threadIdx.x;
    if (r < b && c < a) o[(int64_t)r * a + c] = tile[threadIdx.x][k];
  }
}

static void check_batch(const at::Tensor& x, const char* what) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 3 &&
                  x.size(1) <= 65535 * 32 && x.size(2) <= 65535 * 32 && x.size(0) <= 65535,
              what, ": contiguous bf16 [n, a, b] CUDA batch expected");
}

void ns_normalize(const at::Tensor& x, bool transpose, const at::Tensor& out) {
  check_batch(x, "ns_normalize");
  TORCH_CHECK(x.size(2) % 8 == 0, "ns_normalize: b % 8 == 0");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.numel() == x.numel(),
              "ns_normalize: bf16 output of the same size");
  const int n = x.size(0), a = x.size(1), b = x.size(2);
  if (x.numel() == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const int chunks = (a + NS_ROWS - 1) / NS_ROWS;
  at::Tensor part = at::empty({(int64_t)n * chunks}, x.options().dtype(at::kFloat));
  ns_sumsq_kernel<<<dim3(chunks, n), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), a, b,
                                                  part.data_ptr<float>());
  NG_LAUNCH_CHECK();
  if (transpose) {
    ns_scale_kernel<<<dim3((b + 31) / 32, (a + 31) / 32, n), dim3(32, 8), 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), a, b, part.data_ptr<float>(), chunks, 1,
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  } else {
    const int64_t per = (int64_t)a * b;
    const int64_t bx = std::min<int64_t>((per / 8 + 255) / 256, 64);
    ns_scale_vec_kernel<<<dim3((unsigned)bx, n), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                                               per, part.data_ptr<float>(), chunks,
                                                               reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  }
  NG_LAUNCH_CHECK();
}

void transpose_bf16(const at::Tensor& x, const at::Tensor& out) {
  check_batch(x, "transpose_bf16");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.numel() == x.numel(),
              "transpose_bf16: bf16 output of the same size");
  const int n = x.size(0), a = x.size(1), b = x.size(2);
  if (x.numel() == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  transpose_bf16_kernel<<<dim3((b + 31) / 32, (a + 31) / 32, n), dim3(32, 8), 0,
                          at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), a,
                                                              b, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  NG_LAUNCH_CHECK();
}

}  // namespace ng
