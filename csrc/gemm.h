// Host interface of the tcgen05 GEMM (csrc/gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ng {

// Epilogues fused into the GEMM (see csrc/gemm.cu for the exact formulas).
enum GemmEpi : int {
  EPI_BF16 = 0,        // out = bf16(acc + bias)
  EPI_F32 = 1,         // out (+)= acc in fp32 (weight gradients)
  EPI_AXPBY = 2,       // out = bf16(alpha * acc + beta * res)   (Newton-Schulz steps)
  EPI_GATED = 3,       // y = bf16(acc + bias) -> out2; out = bf16(res + gate[row / rows_per_group] * y)
  EPI_SWIGLU = 4,      // B rows [n, n+128) and [half_n + n, ...): pre -> out2, silu(x1) * x2 -> out
  EPI_SWIGLU_BWD = 5,  // acc = d(act); aux = pre; out = [d x1 | d x2]
};

struct GemmArgs {
  int M = 0, N = 0, K = 0, batch = 1;
  // A: a_mn == 0 -> [M, K] row-major (lda >= K); a_mn == 1 -> [K, M] row-major (lda >= M)
  const void* A = nullptr;
  int64_t lda = 0, a_bs = 0;
  int a_mn = 0;
  // B: b_mn == 0 -> [N, K] row-major; b_mn == 1 -> [K, N] row-major
  const void* B = nullptr;
  int64_t ldb = 0, b_bs = 0;
  int b_mn = 0;
  int64_t b_rows = 0;  // rows of the B tensor map when they differ from N (SwiGLU: 2 * half_n)
  int epi = EPI_BF16;
  void* out = nullptr;
  int64_t ldo = 0, out_bs = 0;
  void* out2 = nullptr;
  int64_t ldo2 = 0;
  const float* bias = nullptr;
  const __nv_bfloat16* res = nullptr;
  int64_t ldr = 0, res_bs = 0;
  const __nv_bfloat16* gate = nullptr;
  int64_t ldg = 0;
  int rows_per_group = 1;
  const int* seg = nullptr;  // optional [M] int32: the gate row of each output row (packed captions); else row / rpg
  const __nv_bfloat16* aux = nullptr;
  int64_t ld_aux = 0;
  int half_n = 0;
  float alpha = 1.f, beta = 0.f;
  int accumulate = 0;
  int k_splits = 1, kb_per_split = 0;
  // MXFP8: A and B are e4m3 (K-major, row strides in bytes) with E8M0 scale factors, one per 32 values along K,
  // in blocks of 128 rows x 4 values: [ceil(rows / 128)][K / 128][512 bytes], byte (r % 32) * 16 + (r / 32 % 4) * 4
  // + (k / 32 % 4) for row r, column k. B's scale factors cover every 128-row block a tile touches.
  int mx = 0;
  const void* sfa = nullptr;
  const void* sfb = nullptr;
  // MX SwiGLU only (optional): also write act in MXFP8 (e4m3 [M, half_n] row-major, scale blocks as above)
  void* act_q = nullptr;
  void* act_sf = nullptr;
  int* err = nullptr;
};

void gemm_launch(const GemmArgs& g, cudaStream_t stream);

CUtensorMap make_tmap_f32_box(const void* ptr, int64_t inner, int64_t outer, int64_t batch, int64_t ld,
                              int64_t bstride, int box_inner, int box_outer);
CUtensorMap make_tmap_bf16(const void* ptr, int64_t inner, int64_t outer, int64_t batch, int64_t ld, int64_t bstride,
                           int box_inner, int box_outer);

}  // namespace ng
