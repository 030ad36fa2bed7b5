// Fixed-order finish of chunk partials inside the kernel that produced them, for sm_100a.
//
// A (chunks x G) grid of CTAs writes partial rows part[(g * chunks + k) * stride + f * C + c] for fields f < NF. The
// last CTA of group g to finish (an atomic ticket per group) adds the group's chunks in chunk order: fields f < NF - 1
// go to per-group outputs out_f[g * ld_f + c]; the last field's group sum goes to scratch[g * C + c], a G-row matrix
// whose column sums the host takes with one small reduction (a single CTA summing all G rows here would be a serial
// tail of tens of microseconds). Which CTA finishes last changes nothing in the sums, so the results are
// deterministic. The ticket is reset by the CTA that took the last one, so the counter table (G ints, zero before
// the first launch) is reused by the next launch on the same stream.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ng {

// Above this many chunks per group the host reduces the partials (two-stage, many CTAs) instead.
constexpr int kFinishMaxChunks = 16;

// Outputs of a finish: up to two per-group fields (null: not wanted), the scratch rows of the last field's group sums
// ([G, C] fp32), and the ticket table (null: no finish in the kernel).
struct FinishArgs {
  float* gout[2];
  int64_t gld[2];
  float* scratch;
  int* cnt;
};

template <int NF>
__device__ __forceinline__ void finish_partials(const float* __restrict__ part, int64_t stride, int C, int chunks,
                                                int g, const FinishArgs& fa) {
  constexpr int NG = NF - 1;  // the last field goes to the scratch rows
  static_assert(NG >= 1 && NG <= 2, "one or two per-group fields");
  int* __restrict__ cnt = fa.cnt;
  float* __restrict__ scratch = fa.scratch;
  __shared__ int s_last;
  __threadfence();  // this CTA's partial row is visible before its ticket
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&cnt[g], 1) == chunks - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float acc[NF];
#pragma unroll
    for (int f = 0; f < NF; ++f) acc[f] = 0.f;
    for (int k = 0; k < chunks; ++k) {
      const float* p = part + (int64_t)(g * chunks + k) * stride + c;
#pragma unroll
      for (int f = 0; f < NF; ++f) acc[f] += __ldcg(p + f * C);
    }
#pragma unroll
    for (int f = 0; f < NG; ++f)
      if (fa.gout[f] != nullptr) fa.gout[f][(int64_t)g * fa.gld[f] + c] = acc[f];
    scratch[(int64_t)g * C + c] = acc[NF - 1];
  }
  if (threadIdx.x == 0) cnt[g] = 0;
}

}  // namespace ng
