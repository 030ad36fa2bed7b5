// Masked multi-head attention, head dim 64, bf16 in / fp32 softmax, forward and backward, for sm_100a.
//
// Keys of sample b are indexed in *storage* order: rows [0, L0) of source 0 then rows [0, L1) of source 1; storage
// key s is valid when s < n0[b] (source 0) or s - L0 < n1[b] (source 1). Key tiles without a valid key are skipped;
// invalid keys inside a tile are masked (and zero-filled on load, so padding never feeds NaN into 0 * x).
// Image blocks: source 0 = image keys (n0 = 256), source 1 = caption keys (n1 = caption length); text blocks: source 0
// = caption keys (n0 = caption length). Reference: the masked SDPA / FA3 joint attention of
// baselines/PixelGen/src/models/transformer/JiT_T2I.py:114-187 and the text attention of :212-265.
//
// This is a flash-attention-2 style kernel on warp-level mma.sync (m16n8k16): 4 warps x 16 query rows per CTA, K/V
// tiles of 64 keys double-buffered with cp.async, 128-byte XOR-swizzled shared-memory tiles read with ldmatrix.
// Backward: delta = rowsum(dO * O); a dK/dV kernel (CTA per key tile, loop over query tiles) and a dQ kernel (CTA per
// query tile, loop over key tiles), so no atomics are needed.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "status.h"

namespace ng {

using bf16 = __nv_bfloat16;

struct AttnParams {
  const bf16* q;
  int64_t ldq;
  const bf16 *k0, *v0, *k1, *v1;
  int64_t ldk0, ldv0, ldk1, ldv1;
  const int *n0, *n1;
  int Lq, L0, L1, H;
  float scale, scale_log2;
  bf16* o;
  int64_t ldo;
  float* lse;
  const bf16* dout;
  int64_t lddo;
  const float* delta;
  bf16* dq;
  int64_t lddq;
  bf16 *dk0, *dv0, *dk1, *dv1;
  int64_t lddk0, lddv0, lddk1, lddv1;
};

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ----------------------------------------------------------------------------------------------------- primitives
__device__ __forceinline__ uint32_t swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Loads the A fragments (4 k-steps of 16) of a 16 x 64 row block starting at row r0 of a swizzled tile.
__device__ __forceinline__ void load_afrag(uint32_t tile, int r0, int lane, uint32_t (&f)[4][4]) {
  const int m = lane >> 3, rr = lane & 7;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int row = r0 + (m & 1) * 8 + rr;
    const int chunk = 2 * ks + (m >> 1);
    ldsm_x4(tile + swz(row, chunk), f[ks][0], f[ks][1], f[ks][2], f[ks][3]);
  }
}

// acc[16 x 64] (+)= A[16 x 64] * T^T where T is a 64 x 64 tile with rows = output columns (keys), cols = reduction.
__device__ __forceinline__ void mma_abt(float (&acc)[8][4], const uint32_t (&a)[4][4], uint32_t tile, int lane) {
  const int m = lane >> 3, rr = lane & 7;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b0, b1, b2, b3;
      const int row = np * 16 + (m >> 1) * 8 + rr;
      const int chunk = 2 * ks + (m & 1);
      ldsm_x4(tile + swz(row, chunk), b0, b1, b2, b3);
      mma16816(acc[2 * np], a[ks], b0, b1);
      mma16816(acc[2 * np + 1], a[ks], b2, b3);
    }
  }
}

// acc[16 x 64] += P[16 x 64] * T where T is a 64 x 64 tile with rows = reduction (keys), cols = output columns;
// P given as fp32 accumulator fragments (8 n-tiles), converted to bf16 A fragments.
__device__ __forceinline__ void mma_pt(float (&acc)[8][4], const float (&p)[8][4], uint32_t tile, int lane) {
  const int m = lane >> 3, rr = lane & 7;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    uint32_t a[4];
    a[0] = pack_bf16(p[2 * ks][0], p[2 * ks][1]);
    a[1] = pack_bf16(p[2 * ks][2], p[2 * ks][3]);
    a[2] = pack_bf16(p[2 * ks + 1][0], p[2 * ks + 1][1]);
    a[3] = pack_bf16(p[2 * ks + 1][2], p[2 * ks + 1][3]);
#pragma unroll
    for (int dp = 0; dp < 4; ++dp) {
      uint32_t b0, b1, b2, b3;
      const int row = ks * 16 + (m & 1) * 8 + rr;
      const int chunk = 2 * dp + (m >> 1);
      ldsm_x4_t(tile + swz(row, chunk), b0, b1, b2, b3);
      mma16816(acc[2 * dp], a, b0, b1);
      mma16816(acc[2 * dp + 1], a, b2, b3);
    }
  }
}

__device__ __forceinline__ void zero8x4(float (&a)[8][4]) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) a[i][j] = 0.f;
}

// storage key s of sample b: valid?
__device__ __forceinline__ bool key_valid(int s, int L0, int L1, int n0b, int n1b) {
  return s < L0 ? (s < n0b) : (s - L0 < n1b && s - L0 < L1);
}
__device__ __forceinline__ bool tile_has_keys(int s0, int L0, int L1, int n0b, int n1b) {
  if (s0 < min(n0b, L0)) return true;
  const int a = max(s0, L0), b = min(s0 + 64, L0 + min(n1b, L1));
  return a < b;
}
__device__ __forceinline__ const bf16* key_ptr(const bf16* src0, int64_t ld0, const bf16* src1, int64_t ld1, int b,
                                               int s, int L0, int L1, int h) {
  if (s < L0) return src0 + ((int64_t)b * L0 + s) * ld0 + h * 64;
  return src1 + ((int64_t)b * L1 + (s - L0)) * ld1 + h * 64;
}

// 64 rows x 128 bytes: thread i loads chunks i, i+128, i+256, i+384.
__device__ __forceinline__ void load_key_tile(uint32_t tile, const bf16* src0, int64_t ld0, const bf16* src1,
                                              int64_t ld1, int b, int s0, int L0, int L1, int n0b, int n1b, int h) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int idx = threadIdx.x + 128 * c;
    const int row = idx >> 3, chunk = idx & 7;
    const int s = s0 + row;
    const bool ok = s < L0 + L1 && key_valid(s, L0, L1, n0b, n1b);
    const bf16* g = ok ? key_ptr(src0, ld0, src1, ld1, b, s, L0, L1, h) + chunk * 8 : src0;
    cp_async16(tile + swz(row, chunk), g, ok);
  }
}
__device__ __forceinline__ void load_q_tile(uint32_t tile, const bf16* src, int64_t ld, int b, int q0, int Lq, int h) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int idx = threadIdx.x + 128 * c;
    const int row = idx >> 3, chunk = idx & 7;
    const bool ok = q0 + row < Lq;
    const bf16* g = ok ? src + ((int64_t)b * Lq + q0 + row) * ld + h * 64 + chunk * 8 : src;
    cp_async16(tile + swz(row, chunk), g, ok);
  }
}

// Stores a warp's 16 x 64 fp32 fragment block (scaled by `mul`) as bf16 rows through a swizzled smem tile.
__device__ __forceinline__ void stage_rows(uint8_t* tile_ptr, int r0, const float (&acc)[8][4], float mul0, float mul1,
                                           int lane) {
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int col = nt * 8 + 2 * t4;
    const int chunk = col >> 3, within = (col & 7) * 2;
    *reinterpret_cast<uint32_t*>(tile_ptr + swz(r0 + g, chunk) + within) = pack_bf16(acc[nt][0] * mul0, acc[nt][1] * mul0);
    *reinterpret_cast<uint32_t*>(tile_ptr + swz(r0 + g + 8, chunk) + within) =
        pack_bf16(acc[nt][2] * mul1, acc[nt][3] * mul1);
  }
}

// ========================================================================================================= forward
__global__ void __launch_bounds__(128) attn_fwd_kernel(const AttnParams p) {
  __shared__ __align__(128) uint8_t sQ[8192];
  __shared__ __align__(128) uint8_t sK[2][8192];
  __shared__ __align__(128) uint8_t sV[2][8192];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int q0 = blockIdx.x * 64;
  const int n0b = p.n0[b], n1b = p.n1 ? p.n1[b] : 0;
  const int nt = (p.L0 + p.L1 + 63) / 64;
  auto next_tile = [&](int k) {
    while (k < nt && !tile_has_keys(k * 64, p.L0, p.L1, n0b, n1b)) ++k;
    return k;
  };
  const uint32_t uQ = smem_u32(sQ), uK0 = smem_u32(sK[0]), uK1 = smem_u32(sK[1]);
  const uint32_t uV0 = smem_u32(sV[0]), uV1 = smem_u32(sV[1]);

  load_q_tile(uQ, p.q, p.ldq, b, q0, p.Lq, h);
  int kt = next_tile(0);
  if (kt < nt) {
    load_key_tile(uK0, p.k0, p.ldk0, p.k1, p.ldk1, b, kt * 64, p.L0, p.L1, n0b, n1b, h);
    load_key_tile(uV0, p.v0, p.ldv0, p.v1, p.ldv1, b, kt * 64, p.L0, p.L1, n0b, n1b, h);
  }
  cp_commit();

  float o[8][4];
  zero8x4(o);
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qf[4][4];
  bool have_q = false;
  for (int it = 0; kt < nt; ++it) {
    const int kn = next_tile(kt + 1);
    const int st = it & 1;
    if (kn < nt) {
      load_key_tile(st ? uK0 : uK1, p.k0, p.ldk0, p.k1, p.ldk1, b, kn * 64, p.L0, p.L1, n0b, n1b, h);
      load_key_tile(st ? uV0 : uV1, p.v0, p.ldv0, p.v1, p.ldv1, b, kn * 64, p.L0, p.L1, n0b, n1b, h);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (!have_q) {
      load_afrag(uQ, warp * 16, lane, qf);
      have_q = true;
    }
    float s[8][4];
    zero8x4(s);
    mma_abt(s, qf, st ? uK1 : uK0, lane);
    // mask + online softmax (rows g and g+8 of this warp)
    const int s0 = kt * 64;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = s0 + n * 8 + 2 * t4 + (e & 1);
        const bool ok = key < p.L0 + p.L1 && key_valid(key, p.L0, p.L1, n0b, n1b);
        s[n][e] = ok ? s[n][e] * p.scale_log2 : -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[n][e]);
      }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(m_r[r], mx[r]);
      corr[r] = exp2f(m_r[r] - mnew);
      m_r[r] = mnew;
      l_r[r] *= corr[r];
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[n][e] = exp2f(s[n][e] - m_r[e >> 1]);
        l_r[e >> 1] += s[n][e];
      }
    }
    mma_pt(o, s, st ? uV1 : uV0, lane);
    __syncthreads();
    kt = kn;
  }
  cp_wait<0>();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  const float inv0 = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f, inv1 = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
  __syncthreads();
  stage_rows(sQ, warp * 16, o, inv0, inv1, lane);
  if (t4 == 0) {
    const int qa = q0 + warp * 16 + g, qb = qa + 8;
    float* lp = p.lse + ((int64_t)b * p.H + h) * p.Lq;
    if (qa < p.Lq) lp[qa] = (m_r[0] + log2f(l_r[0])) * kLn2;
    if (qb < p.Lq) lp[qb] = (m_r[1] + log2f(l_r[1])) * kLn2;
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int idx = threadIdx.x + 128 * c;
    const int row = idx >> 3, chunk = idx & 7;
    if (q0 + row < p.Lq)
      *reinterpret_cast<uint4*>(p.o + ((int64_t)b * p.Lq + q0 + row) * p.ldo + h * 64 + chunk * 8) =
          *reinterpret_cast<const uint4*>(sQ + swz(row, chunk));
  }
}

// ======================================================================================================== backward
// delta[b, h, q] = sum_d dO * O
__global__ void attn_delta_kernel(const bf16* __restrict__ dout, int64_t lddo, const bf16* __restrict__ o, int64_t ldo,
                                  float* __restrict__ delta, int rows, int Lq, int H) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (int64_t)rows * H) return;
  const int row = (int)(t / H), h = (int)(t - (int64_t)row * H);
  const uint4* a = reinterpret_cast<const uint4*>(dout + row * lddo + h * 64);
  const uint4* c = reinterpret_cast<const uint4*>(o + row * ldo + h * 64);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 x = a[i], y = c[i];
    acc += bf16_bits_lo(x.x) * bf16_bits_lo(y.x) + bf16_bits_hi(x.x) * bf16_bits_hi(y.x);
    acc += bf16_bits_lo(x.y) * bf16_bits_lo(y.y) + bf16_bits_hi(x.y) * bf16_bits_hi(y.y);
    acc += bf16_bits_lo(x.z) * bf16_bits_lo(y.z) + bf16_bits_hi(x.z) * bf16_bits_hi(y.z);
    acc += bf16_bits_lo(x.w) * bf16_bits_lo(y.w) + bf16_bits_hi(x.w) * bf16_bits_hi(y.w);
  }
  const int b = row / Lq, q = row - b * Lq;
  delta[((int64_t)b * H + h) * Lq + q] = acc;
}

// dK, dV for one storage key tile; loops over the query tiles.
__global__ void __launch_bounds__(128) attn_bwd_dkdv_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sK = smem;
  uint8_t* sV = smem + 8192;
  uint8_t* sQ = smem + 16384;             // [2][8192]
  uint8_t* sD = smem + 32768;             // dO [2][8192]
  float* sL = reinterpret_cast<float*>(smem + 49152);  // lse*log2e [2][64]
  float* sDl = sL + 128;                               // delta [2][64]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int s0 = blockIdx.x * 64;
  const int n0b = p.n0[b], n1b = p.n1 ? p.n1[b] : 0;
  const int Ls = p.L0 + p.L1;
  if (!tile_has_keys(s0, p.L0, p.L1, n0b, n1b)) {
    // no valid key: zero gradients for the rows of this tile
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int idx = threadIdx.x + 128 * c;
      const int row = idx >> 3, chunk = idx & 7;
      const int s = s0 + row;
      if (s >= Ls) continue;
      bf16* dk = s < p.L0 ? p.dk0 + ((int64_t)b * p.L0 + s) * p.lddk0 : p.dk1 + ((int64_t)b * p.L1 + s - p.L0) * p.lddk1;
      bf16* dv = s < p.L0 ? p.dv0 + ((int64_t)b * p.L0 + s) * p.lddv0 : p.dv1 + ((int64_t)b * p.L1 + s - p.L0) * p.lddv1;
      *reinterpret_cast<uint4*>(dk + h * 64 + chunk * 8) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(dv + h * 64 + chunk * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const uint32_t uK = smem_u32(sK), uV = smem_u32(sV), uQ = smem_u32(sQ), uD = smem_u32(sD);
  load_key_tile(uK, p.k0, p.ldk0, p.k1, p.ldk1, b, s0, p.L0, p.L1, n0b, n1b, h);
  load_key_tile(uV, p.v0, p.ldv0, p.v1, p.ldv1, b, s0, p.L0, p.L1, n0b, n1b, h);
  const int nq = (p.Lq + 63) / 64;
  const float* lse_bh = p.lse + ((int64_t)b * p.H + h) * p.Lq;
  const float* del_bh = p.delta + ((int64_t)b * p.H + h) * p.Lq;
  auto load_q = [&](int qt, int st) {
    load_q_tile(uQ + st * 8192, p.q, p.ldq, b, qt * 64, p.Lq, h);
    load_q_tile(uD + st * 8192, p.dout, p.lddo, b, qt * 64, p.Lq, h);
    if (threadIdx.x < 64) {
      const int q = qt * 64 + threadIdx.x;
      sL[st * 64 + threadIdx.x] = q < p.Lq ? lse_bh[q] * kLog2e : INFINITY;
      sDl[st * 64 + threadIdx.x] = q < p.Lq ? del_bh[q] : 0.f;
    }
  };
  load_q(0, 0);
  cp_commit();
  float dv[8][4], dk[8][4];
  zero8x4(dv);
  zero8x4(dk);
  uint32_t kf[4][4], vf[4][4];
  // key rows of this thread (for masking P^T rows)
  const int ka = s0 + warp * 16 + g, kb = ka + 8;
  const bool va = ka < Ls && key_valid(ka, p.L0, p.L1, n0b, n1b);
  const bool vb = kb < Ls && key_valid(kb, p.L0, p.L1, n0b, n1b);
  for (int qt = 0; qt < nq; ++qt) {
    const int st = qt & 1;
    __syncthreads();  // the other stage is free (previous iteration done with it)
    if (qt + 1 < nq) load_q(qt + 1, st ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (qt == 0) {
      load_afrag(uK, warp * 16, lane, kf);
      load_afrag(uV, warp * 16, lane, vf);
    }
    const uint32_t tQ = uQ + st * 8192, tD = uD + st * 8192;
    // S^T = K_w Q^T  (16 keys x 64 queries)
    float sT[8][4];
    zero8x4(sT);
    mma_abt(sT, kf, tQ, lane);
    // P^T
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = n * 8 + 2 * t4 + (e & 1);
        const bool ok = (e < 2) ? va : vb;
        sT[n][e] = ok ? exp2f(sT[n][e] * p.scale_log2 - sL[st * 64 + qc]) : 0.f;
      }
    // dV += P^T dO
    mma_pt(dv, sT, tD, lane);
    // dP^T = V_w dO^T
    float dpT[8][4];
    zero8x4(dpT);
    mma_abt(dpT, vf, tD, lane);
    // dS^T = P^T (dP^T - delta)
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = n * 8 + 2 * t4 + (e & 1);
        dpT[n][e] = sT[n][e] * (dpT[n][e] - sDl[st * 64 + qc]);
      }
    // dK += dS^T Q
    mma_pt(dk, dpT, tQ, lane);
  }
  cp_wait<0>();
  __syncthreads();
  // write dK (scaled) and dV through smem staging (reuse sQ stage 0 / stage 1)
  stage_rows(sQ, warp * 16, dk, p.scale, p.scale, lane);
  stage_rows(sQ + 8192, warp * 16, dv, 1.f, 1.f, lane);
  __syncthreads();
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int idx = threadIdx.x + 128 * c;
    const int row = idx >> 3, chunk = idx & 7;
    const int s = s0 + row;
    if (s >= Ls) continue;
    bf16* dkp = s < p.L0 ? p.dk0 + ((int64_t)b * p.L0 + s) * p.lddk0 : p.dk1 + ((int64_t)b * p.L1 + s - p.L0) * p.lddk1;
    bf16* dvp = s < p.L0 ? p.dv0 + ((int64_t)b * p.L0 + s) * p.lddv0 : p.dv1 + ((int64_t)b * p.L1 + s - p.L0) * p.lddv1;
    *reinterpret_cast<uint4*>(dkp + h * 64 + chunk * 8) = *reinterpret_cast<const uint4*>(sQ + swz(row, chunk));
    *reinterpret_cast<uint4*>(dvp + h * 64 + chunk * 8) = *reinterpret_cast<const uint4*>(sQ + 8192 + swz(row, chunk));
  }
}

// dQ for one query tile; loops over the valid key tiles.
__global__ void __launch_bounds__(128) attn_bwd_dq_kernel(const AttnParams p) {
  __shared__ __align__(128) uint8_t sQ[8192];
  __shared__ __align__(128) uint8_t sO[8192];  // dO tile, later the output staging
  __shared__ __align__(128) uint8_t sK[2][8192];
  __shared__ __align__(128) uint8_t sV[2][8192];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int q0 = blockIdx.x * 64;
  const int n0b = p.n0[b], n1b = p.n1 ? p.n1[b] : 0;
  const int nt = (p.L0 + p.L1 + 63) / 64;
  auto next_tile = [&](int k) {
    while (k < nt && !tile_has_keys(k * 64, p.L0, p.L1, n0b, n1b)) ++k;
    return k;
  };
  const uint32_t uQ = smem_u32(sQ), uO = smem_u32(sO);
  const uint32_t uK0 = smem_u32(sK[0]), uK1 = smem_u32(sK[1]), uV0 = smem_u32(sV[0]), uV1 = smem_u32(sV[1]);
  load_q_tile(uQ, p.q, p.ldq, b, q0, p.Lq, h);
  load_q_tile(uO, p.dout, p.lddo, b, q0, p.Lq, h);
  int kt = next_tile(0);
  if (kt < nt) {
    load_key_tile(uK0, p.k0, p.ldk0, p.k1, p.ldk1, b, kt * 64, p.L0, p.L1, n0b, n1b, h);
    load_key_tile(uV0, p.v0, p.ldv0, p.v1, p.ldv1, b, kt * 64, p.L0, p.L1, n0b, n1b, h);
  }
  cp_commit();
  const int qa = q0 + warp * 16 + g, qb = qa + 8;
  const float* lse_bh = p.lse + ((int64_t)b * p.H + h) * p.Lq;
  const float* del_bh = p.delta + ((int64_t)b * p.H + h) * p.Lq;
  const float la = qa < p.Lq ? lse_bh[qa] * kLog2e : INFINITY, lb = qb < p.Lq ? lse_bh[qb] * kLog2e : INFINITY;
  const float da = qa < p.Lq ? del_bh[qa] : 0.f, db = qb < p.Lq ? del_bh[qb] : 0.f;
  float dq[8][4];
  zero8x4(dq);
  uint32_t qf[4][4], of[4][4];
  bool have = false;
  for (int it = 0; kt < nt; ++it) {
    const int kn = next_tile(kt + 1);
    const int st = it & 1;
    if (kn < nt) {
      load_key_tile(st ? uK0 : uK1, p.k0, p.ldk0, p.k1, p.ldk1, b, kn * 64, p.L0, p.L1, n0b, n1b, h);
      load_key_tile(st ? uV0 : uV1, p.v0, p.ldv0, p.v1, p.ldv1, b, kn * 64, p.L0, p.L1, n0b, n1b, h);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (!have) {
      load_afrag(uQ, warp * 16, lane, qf);
      load_afrag(uO, warp * 16, lane, of);
      have = true;
    }
    float s[8][4];
    zero8x4(s);
    mma_abt(s, qf, st ? uK1 : uK0, lane);
    const int s0 = kt * 64;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = s0 + n * 8 + 2 * t4 + (e & 1);
        const bool ok = key < p.L0 + p.L1 && key_valid(key, p.L0, p.L1, n0b, n1b);
        s[n][e] = ok ? exp2f(s[n][e] * p.scale_log2 - ((e < 2) ? la : lb)) : 0.f;
      }
    float dp[8][4];
    zero8x4(dp);
    mma_abt(dp, of, st ? uV1 : uV0, lane);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) dp[n][e] = s[n][e] * (dp[n][e] - ((e < 2) ? da : db));
    mma_pt(dq, dp, st ? uK1 : uK0, lane);
    __syncthreads();
    kt = kn;
  }
  cp_wait<0>();
  __syncthreads();
  stage_rows(sO, warp * 16, dq, p.scale, p.scale, lane);
  __syncthreads();
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int idx = threadIdx.x + 128 * c;
    const int row = idx >> 3, chunk = idx & 7;
    if (q0 + row < p.Lq)
      *reinterpret_cast<uint4*>(p.dq + ((int64_t)b * p.Lq + q0 + row) * p.lddq + h * 64 + chunk * 8) =
          *reinterpret_cast<const uint4*>(sO + swz(row, chunk));
  }
}

// ====================================================================================================== torch glue
static const bf16* bp(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<const bf16*>(t->data_ptr()) : nullptr;
}
static bf16* bpm(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<bf16*>(t->data_ptr()) : nullptr;
}
static int64_t ldv(const c10::optional<at::Tensor>& t) { return (t.has_value() && t->defined()) ? t->stride(0) : 0; }

static void check_view(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.stride(1) == 1 && t.scalar_type() == at::kBFloat16, name,
              ": 2-D bf16 CUDA view with unit last stride expected");
  TORCH_CHECK(t.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name,
              ": rows must be 16-byte aligned");
}

static AttnParams make_params(const at::Tensor& q, const at::Tensor& k0, const at::Tensor& v0,
                              const c10::optional<at::Tensor>& k1, const c10::optional<at::Tensor>& v1,
                              const at::Tensor& n0, const at::Tensor& n1, int64_t Lq, int64_t L0, int64_t L1,
                              double scale) {
  check_view(q, "q");
  check_view(k0, "k0");
  check_view(v0, "v0");
  TORCH_CHECK(q.size(1) % 64 == 0, "head dim 64 expected");
  TORCH_CHECK(n0.scalar_type() == at::kInt && n1.scalar_type() == at::kInt, "int32 key counts expected");
  AttnParams p{};
  p.q = reinterpret_cast<const bf16*>(q.data_ptr());
  p.ldq = q.stride(0);
  p.k0 = reinterpret_cast<const bf16*>(k0.data_ptr());
  p.v0 = reinterpret_cast<const bf16*>(v0.data_ptr());
  p.ldk0 = k0.stride(0);
  p.ldv0 = v0.stride(0);
  p.k1 = bp(k1);
  p.v1 = bp(v1);
  p.ldk1 = ldv(k1);
  p.ldv1 = ldv(v1);
  if (p.k1 == nullptr) L1 = 0;
  p.n0 = n0.data_ptr<int>();
  p.n1 = n1.data_ptr<int>();
  p.Lq = (int)Lq;
  p.L0 = (int)L0;
  p.L1 = (int)L1;
  p.H = (int)(q.size(1) / 64);
  p.scale = (float)scale;
  p.scale_log2 = (float)scale * kLog2e;
  return p;
}

void attn_fwd(const at::Tensor& q, const at::Tensor& k0, const at::Tensor& v0, const c10::optional<at::Tensor>& k1,
              const c10::optional<at::Tensor>& v1, const at::Tensor& n0, const at::Tensor& n1, const at::Tensor& o,
              const at::Tensor& lse, int64_t Lq, int64_t L0, int64_t L1, double scale) {
  const at::cuda::CUDAGuard guard(q.device());
  AttnParams p = make_params(q, k0, v0, k1, v1, n0, n1, Lq, L0, L1, scale);
  check_view(o, "o");
  p.o = reinterpret_cast<bf16*>(o.data_ptr());
  p.ldo = o.stride(0);
  p.lse = lse.data_ptr<float>();
  const int B = (int)(q.size(0) / Lq);
  dim3 grid((unsigned)((Lq + 63) / 64), (unsigned)(B * p.H));
  attn_fwd_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  NG_LAUNCH_CHECK();
}

void attn_delta(const bf16* dout, int64_t lddo, const bf16* o, int64_t ldo, float* delta, int rows, int Lq, int H,
                cudaStream_t s) {
  const int64_t n = (int64_t)rows * H;
  attn_delta_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dout, lddo, o, ldo, delta, rows, Lq, H);
  NG_LAUNCH_CHECK();
}

void attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k0, const at::Tensor& v0,
              const c10::optional<at::Tensor>& k1, const c10::optional<at::Tensor>& v1, const at::Tensor& n0,
              const at::Tensor& n1, const at::Tensor& o, const at::Tensor& lse, const at::Tensor& dq,
              const at::Tensor& dk0, const at::Tensor& dv0, const c10::optional<at::Tensor>& dk1,
              const c10::optional<at::Tensor>& dv1, int64_t Lq, int64_t L0, int64_t L1, double scale) {
  const at::cuda::CUDAGuard guard(q.device());
  AttnParams p = make_params(q, k0, v0, k1, v1, n0, n1, Lq, L0, L1, scale);
  check_view(dout, "dout");
  check_view(o, "o");
  check_view(dq, "dq");
  check_view(dk0, "dk0");
  check_view(dv0, "dv0");
  p.o = reinterpret_cast<bf16*>(o.data_ptr());
  p.ldo = o.stride(0);
  p.lse = lse.data_ptr<float>();
  p.dout = reinterpret_cast<const bf16*>(dout.data_ptr());
  p.lddo = dout.stride(0);
  p.dq = reinterpret_cast<bf16*>(dq.data_ptr());
  p.lddq = dq.stride(0);
  p.dk0 = reinterpret_cast<bf16*>(dk0.data_ptr());
  p.lddk0 = dk0.stride(0);
  p.dv0 = reinterpret_cast<bf16*>(dv0.data_ptr());
  p.lddv0 = dv0.stride(0);
  p.dk1 = bpm(dk1);
  p.lddk1 = ldv(dk1);
  p.dv1 = bpm(dv1);
  p.lddv1 = ldv(dv1);
  const int B = (int)(q.size(0) / Lq);
  auto s = at::cuda::getCurrentCUDAStream();
  at::Tensor delta = at::empty({(int64_t)B, p.H, Lq}, q.options().dtype(at::kFloat));
  p.delta = delta.data_ptr<float>();
  const int64_t n = q.size(0) * (int64_t)p.H;
  attn_delta_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(p.dout, p.lddo, p.o, p.ldo, delta.data_ptr<float>(),
                                                                 (int)q.size(0), (int)Lq, p.H);
  NG_LAUNCH_CHECK();
  constexpr int kDkdvSmem = 49152 + 4 * 128 * 4;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attn_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDkdvSmem);
    attr = true;
  }
  dim3 g1((unsigned)((p.L0 + p.L1 + 63) / 64), (unsigned)(B * p.H));
  attn_bwd_dkdv_kernel<<<g1, 128, kDkdvSmem, s>>>(p);
  NG_LAUNCH_CHECK();
  dim3 g2((unsigned)((Lq + 63) / 64), (unsigned)(B * p.H));
  attn_bwd_dq_kernel<<<g2, 128, 0, s>>>(p);
  NG_LAUNCH_CHECK();
}

}  // namespace ng
