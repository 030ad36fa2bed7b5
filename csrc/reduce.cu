// Deterministic column sums for the backward passes (bias gradients, norm-weight gradients, per-sample modulation
// gradients), for sm_100a.
//   colsum: out[c] (+)= sum_r src[r * ld + c] over rows, fp32 or bf16 source. Two stages: S row ranges x 32-column
//           blocks write fp32 partials (lanes over columns: coalesced 128-byte rows; 8 warps over rows, combined in a
//           fixed order through shared memory), then one thread per column adds the S partials in order.
//   group_sum: out[g * ldo + c] = sum_{k < chunks} part[(g * chunks + k) * stride + c] (the chunk partials of one
//           modulation group, e.g. one sample).
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAGraphsUtils.cuh>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>

#include "common.cuh"
#include "reduce.h"
#include "status.h"

namespace ng {

__device__ __forceinline__ float ld_as_f(const float* p) { return *p; }
__device__ __forceinline__ float ld_as_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }

template <typename T>
__global__ void __launch_bounds__(256) colsum_partial_kernel(const T* __restrict__ src, int64_t rows, int C, int64_t ld,
                                                             float* __restrict__ part) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, wy = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int S = gridDim.y, s = blockIdx.y;
  const int64_t per = (rows + S - 1) / S;
  const int64_t r0 = s * per, r1 = min(rows, r0 + per);
  float acc = 0.f;
  if (c < C)
    for (int64_t r = r0 + wy; r < r1; r += 8) acc += ld_as_f(src + r * ld + c);
  red[wy][lane] = acc;
  __syncthreads();
  if (wy == 0 && c < C) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][lane];
    part[(int64_t)s * C + c] = t;
  }
}

__global__ void colsum_final_kernel(const float* __restrict__ part, int S, int C, float* __restrict__ out, int acc) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float t = 0.f;
  for (int s = 0; s < S; ++s) t += part[(int64_t)s * C + c];
  out[c] = acc ? out[c] + t : t;
}

__global__ void group_sum_kernel(const float* __restrict__ part, int chunks, int C, int64_t stride, float* out,
                                 int64_t ldo) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x, g = blockIdx.y;
  if (c >= C) return;
  float t = 0.f;
  for (int k = 0; k < chunks; ++k) t += part[(int64_t)(g * chunks + k) * stride + c];
  out[(int64_t)g * ldo + c] = t;
}

void colsum_launch(const void* src, bool src_bf16, int64_t rows, int C, int64_t ld, float* out, bool accumulate,
                   cudaStream_t stream) {
  if (rows <= 0 || C <= 0) return;
  const int S = (int)std::min<int64_t>(std::max<int64_t>(1, rows / 64), 256);
  at::Tensor part = at::empty({(int64_t)S * C}, at::TensorOptions().device(at::kCUDA).dtype(at::kFloat));
  const dim3 grid((C + 31) / 32, S);
  if (src_bf16)
    colsum_partial_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), rows, C,
                                                                    ld, part.data_ptr<float>());
  else
    colsum_partial_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(src), rows, C, ld,
                                                            part.data_ptr<float>());
  NG_LAUNCH_CHECK();
  colsum_final_kernel<<<(C + 255) / 256, 256, 0, stream>>>(part.data_ptr<float>(), S, C, out, accumulate ? 1 : 0);
  NG_LAUNCH_CHECK();
}

void group_sum_launch(const float* part, int G, int chunks, int C, int64_t stride, float* out, int64_t ldo,
                      cudaStream_t stream) {
  if (out == nullptr || G <= 0) return;
  group_sum_kernel<<<dim3((C + 255) / 256, G), 256, 0, stream>>>(part, chunks, C, stride, out, ldo);
  NG_LAUNCH_CHECK();
}

int* finish_counters(cudaStream_t stream, int n) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, std::pair<int*, int>> tables;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto& t = tables[{dev, stream}];
  if (t.second < n) {
    at::cuda::assertNotCapturing("finish_counters: allocating the ticket table");
    int* p = nullptr;
    const int cap = std::max(n, 4096);
    TORCH_CHECK(cudaMalloc(&p, cap * sizeof(int)) == cudaSuccess, "finish_counters: cudaMalloc failed");
    TORCH_CHECK(cudaMemsetAsync(p, 0, cap * sizeof(int), stream) == cudaSuccess, "finish_counters: memset failed");
    if (t.first != nullptr) {
      cudaStreamSynchronize(stream);  // the old table's last user on this stream has finished
      cudaFree(t.first);
    }
    t = {p, cap};
  }
  return t.first;
}

// torch: out (+)= column sums of src [rows, C] (fp32 or bf16, unit column stride)
void colsum(const at::Tensor& src, const at::Tensor& out, bool accumulate) {
  TORCH_CHECK(src.is_cuda() && src.dim() == 2 && src.stride(1) == 1, "colsum: 2-D CUDA source with unit column stride");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == src.size(1),
              "colsum: fp32 output of C values");
  const at::cuda::CUDAGuard guard(src.device());
  colsum_launch(src.data_ptr(), src.scalar_type() == at::kBFloat16, src.size(0), (int)src.size(1), src.stride(0),
                out.data_ptr<float>(), accumulate, at::cuda::getCurrentCUDAStream());
}

}  // namespace ng
