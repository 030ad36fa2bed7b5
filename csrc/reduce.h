// Deterministic column reductions shared by the backward kernels (csrc/reduce.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ng {
// out[c] (+)= sum over rows of src[r * ld + c]; src fp32 or bf16. Allocates an S x C fp32 partial buffer.
void colsum_launch(const void* src, bool src_bf16, int64_t rows, int C, int64_t ld, float* out, bool accumulate,
                   cudaStream_t stream);
// out[g * ldo + c] = sum_{k < chunks} part[(g * chunks + k) * stride + c]; no-op when out is null.
void group_sum_launch(const float* part, int G, int chunks, int C, int64_t stride, float* out, int64_t ldo,
                      cudaStream_t stream);
// The ticket table of finish_partials (csrc/finish.cuh) for launches on `stream`: at least n zeroed ints, kept per
// (device, stream) and reused (every finishing kernel leaves it zeroed).
int* finish_counters(cudaStream_t stream, int n);
}  // namespace ng
