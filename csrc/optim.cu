// Table-driven Muon kernels: one launch for work that the optimizer would otherwise issue once per matrix unit.
//
// Role of the reference's Muon-add lever (baselines/PixelGen/src/optim/muon_add.py:9-35: `W += alpha_k O_k` for every
// unit from a device pointer table, one Triton launch) and of the per-unit Nesterov inputs stacked for the batched
// Newton-Schulz (baselines/PixelGen/src/optim/muon.py:150-216). A d12 model has 219 units (q, k, v, k_y, v_y, proj, the
// two SwiGLU halves, w3 and the six adaLN parts of every block); issued one by one, their lerps, copies and adds are
// ~660 tiny launches per step that leave the GPU waiting on the host.
//
// muon_gather: rows [dst fp32*, grad fp32*, momentum fp32*, numel]: dst = nesterov ? lerp(grad, momentum, beta)
//              : momentum, with torch.lerp's formula (the end-anchored form for weights >= 0.5).
// muon_apply:  rows [param fp32*, update bf16*, numel, coef (fp32 bits)]: param = param * decay + coef * update.
// numel is a multiple of 4 and every pointer is 16-byte aligned (row slices of contiguous matrices); the host checks.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include "status.h"

namespace ng {

__device__ __forceinline__ float lerp_torch(float a, float b, float w) {
  return fabsf(w) < 0.5f ? a + w * (b - a) : b - (b - a) * (1.0f - w);
}

__global__ void muon_gather_kernel(const int64_t* __restrict__ tab, float beta, int nesterov) {
  const int64_t* r = tab + (int64_t)blockIdx.y * 4;
  float4* dst = reinterpret_cast<float4*>(r[0]);
  const float4* g = reinterpret_cast<const float4*>(r[1]);
  const float4* m = reinterpret_cast<const float4*>(r[2]);
  const int64_t n4 = r[3] / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 mv = m[i];
    if (nesterov) {
      const float4 gv = g[i];
      dst[i] = make_float4(lerp_torch(gv.x, mv.x, beta), lerp_torch(gv.y, mv.y, beta), lerp_torch(gv.z, mv.z, beta),
                           lerp_torch(gv.w, mv.w, beta));
    } else {
      dst[i] = mv;
    }
  }
}

__global__ void muon_apply_kernel(const int64_t* __restrict__ tab, float decay) {
  const int64_t* r = tab + (int64_t)blockIdx.y * 4;
  float4* p = reinterpret_cast<float4*>(r[0]);
  const uint2* u = reinterpret_cast<const uint2*>(r[1]);  // 4 bf16
  const int64_t n4 = r[2] / 4;
  const float coef = __int_as_float((int)r[3]);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const uint2 w = u[i];
    float4 v = p[i];
    v.x = v.x * decay + coef * __uint_as_float(w.x << 16);
    v.y = v.y * decay + coef * __uint_as_float(w.x & 0xFFFF0000u);
    v.z = v.z * decay + coef * __uint_as_float(w.y << 16);
    v.w = v.w * decay + coef * __uint_as_float(w.y & 0xFFFF0000u);
    p[i] = v;
  }
}

static dim3 table_grid(const at::Tensor& tab, int64_t max_numel) {
  TORCH_CHECK(tab.is_cuda() && tab.scalar_type() == at::kLong && tab.dim() == 2 && tab.size(1) == 4 &&
                  tab.is_contiguous(),
              "muon table: [rows, 4] int64 CUDA tensor expected");
  TORCH_CHECK(tab.size(0) <= 65535, "muon table: at most 65535 rows");
  const int64_t blocks = std::min<int64_t>((max_numel / 4 + 255) / 256, 64);
  return dim3((unsigned)std::max<int64_t>(blocks, 1), (unsigned)tab.size(0));
}

void muon_gather(const at::Tensor& tab, double beta, bool nesterov, int64_t max_numel) {
  if (tab.size(0) == 0) return;
  const at::cuda::CUDAGuard guard(tab.device());
  muon_gather_kernel<<<table_grid(tab, max_numel), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      tab.data_ptr<int64_t>(), (float)beta, nesterov ? 1 : 0);
  NG_LAUNCH_CHECK();
}

void muon_apply(const at::Tensor& tab, double decay, int64_t max_numel) {
  if (tab.size(0) == 0) return;
  const at::cuda::CUDAGuard guard(tab.device());
  muon_apply_kernel<<<table_grid(tab, max_numel), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      tab.data_ptr<int64_t>(), (float)decay);
  NG_LAUNCH_CHECK();
}

}  // namespace ng
