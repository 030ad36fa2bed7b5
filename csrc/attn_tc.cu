// Masked multi-head attention forward on the 5th-generation tensor cores (tcgen05 + TMEM), head dim 64, for sm_100a.
//
// One CTA per (128 queries, sample, head). Keys are visited in 128-key tiles of the storage order (rows [0, L0) of
// source 0, then rows [0, L1) of source 1; the key-validity rule is that of csrc/attention.cu); tiles without a valid
// key are skipped. Per tile j:
//   MMA warp      S_j = Q K_j^T        (M=128 queries, N=128 keys, K=64) into TMEM buffer j % 2
//                 O  += P_{j-1} V_{j-1}  (M=128, N=64, K=128; P from shared memory, V as an MN-major operand)
//   softmax warps (a thread per query row) read S_j from TMEM, mask, online-softmax update (running max m, sum l),
//                 rescale O in TMEM by exp(m_old - m_new), write P_j (bf16, 128-byte swizzle) to shared memory
//   TMA warp      K_j, V_j (one 3-D box each: rows past a sample's length are zero-filled, never the next sample's)
// S_{j+1} is computed while the softmax works on S_j. The epilogue divides O by l, stores it and the log-sum-exp.
// Reference: the joint image/caption attention of baselines/PixelGen/src/models/transformer/JiT_T2I.py:114-187.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "gemm.h"
#include "status.h"

namespace ng {

using bf16 = __nv_bfloat16;

namespace atc {
constexpr int BQ = 128, BKV = 128, D = 64;
constexpr int THREADS = 192;  // warp 0 TMA, warp 1 MMA, warps 2..5 softmax
constexpr int Q_BYTES = BQ * D * 2;        // 16 KiB
constexpr int KV_BYTES = BKV * D * 2;      // 16 KiB each of K and V
constexpr int P_BYTES = BQ * BKV * 2;      // 32 KiB (two 64-key swizzle atoms)
constexpr int SMEM = Q_BYTES + 2 * 2 * KV_BYTES + 2 * P_BYTES + 1024 + 256;
constexpr uint32_t TMEM_COLS = 512;        // S0 [0,128), S1 [128,256), O [256,320)
constexpr uint32_t O_COL = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
}  // namespace atc

struct AttnTcParams {
  const int *n0, *n1;
  int Lq, L0, L1, H;
  int nt0, nt1;  // 128-key tiles of each source
  float scale_log2;
  bf16* o;
  int64_t ldo;
  float* lse;
  int* err;
};

__device__ __forceinline__ bool atc_tile_live(int j, const AttnTcParams& p, int n0b, int n1b) {
  return j < p.nt0 ? (j * atc::BKV < n0b) : ((j - p.nt0) * atc::BKV < n1b);
}
__device__ __forceinline__ bool atc_key_valid(int j, int c, const AttnTcParams& p, int n0b, int n1b) {
  if (j < p.nt0) {
    const int s = j * atc::BKV + c;
    return s < n0b && s < p.L0;
  }
  const int s = (j - p.nt0) * atc::BKV + c;
  return s < n1b && s < p.L1;
}

__global__ void __launch_bounds__(atc::THREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK0,
                       const __grid_constant__ CUtensorMap tmV0, const __grid_constant__ CUtensorMap tmK1,
                       const __grid_constant__ CUtensorMap tmV1, const AttnTcParams p) {
  using namespace atc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + Q_BYTES;                 // stage s: K at s * 2 * KV_BYTES, V after it
  uint8_t* sP = sKV + 4 * KV_BYTES;            // buffer b at b * P_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* p_full = bars + 7;    // [2]
  uint64_t* o_done = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int q0 = blockIdx.x * BQ;
  const int n0b = p.n0[b], n1b = p.n1 ? p.n1[b] : 0;
  const int nt = p.nt0 + p.nt1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // --------------------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, Q_BYTES);
      tma_load_3d(&tmQ, q_full, sQ, h * D, q0, b);
      int it = 0;
      for (int j = 0; j < nt; ++j) {
        if (!atc_tile_live(j, p, n0b, n1b)) continue;
        const int st = it & 1;
        if (!mbar_wait(&kv_empty[st], ((it >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        uint8_t* k = sKV + st * 2 * KV_BYTES;
        mbar_arrive_expect_tx(&kv_full[st], 2 * KV_BYTES);
        if (j < p.nt0) {
          tma_load_3d(&tmK0, &kv_full[st], k, h * D, j * BKV, b);
          tma_load_3d(&tmV0, &kv_full[st], k + KV_BYTES, h * D, j * BKV, b);
        } else {
          tma_load_3d(&tmK1, &kv_full[st], k, h * D, (j - p.nt0) * BKV, b);
          tma_load_3d(&tmV1, &kv_full[st], k + KV_BYTES, h * D, (j - p.nt0) * BKV, b);
        }
        ++it;
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(BQ, BKV, 0, 0);
      constexpr uint32_t idesc_o = idesc_bf16_f32(BQ, D, 0, 1);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err, kErrWaitFull);
      const uint32_t aq = smem_u32(sQ);
      int it = 0;
      // issue S for live tile `it` (its K/V are in stage it % 2)
      auto issue_s = [&](int i) {
        const int st = i & 1;
        if (!mbar_wait(&kv_full[st], (i >> 1) & 1, abort_flag, p.err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t kb = smem_u32(sKV + st * 2 * KV_BYTES);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          umma_f16(tmem + st * BKV, smem_desc_sw128(aq + k * 32, 16, 1024), smem_desc_sw128(kb + k * 32, 16, 1024),
                   idesc_s, k != 0 ? 1u : 0u);
        umma_commit(&s_full[st]);
        return true;
      };
      auto issue_pv = [&](int i) {
        const int st = i & 1;
        if (!mbar_wait(&p_full[st], (i >> 1) & 1, abort_flag, p.err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t pa = smem_u32(sP + st * P_BYTES);
        const uint32_t vb = smem_u32(sKV + st * 2 * KV_BYTES + KV_BYTES);
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k)
          umma_f16(tmem + O_COL, smem_desc_sw128(pa + (k >> 2) * (P_BYTES / 2) + (k & 3) * 32, 16, 1024),
                   smem_desc_sw128(vb + k * 2048, 8192, 1024), idesc_o, (i != 0 || k != 0) ? 1u : 0u);
        umma_commit(o_done);
        umma_commit(&kv_empty[st]);
        return true;
      };
      int nlive = 0;
      for (int j = 0; j < nt; ++j) nlive += atc_tile_live(j, p, n0b, n1b) ? 1 : 0;
      for (it = 0; ok && it < nlive; ++it) {
        if (!issue_s(it)) break;
        if (it >= 1 && !issue_pv(it - 1)) break;
      }
      if (ok && it == nlive && nlive > 0) issue_pv(nlive - 1);
    }
  } else {
    // --------------------------------------------------------------------------------------- softmax / epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;  // query row within the tile
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    float m = -INFINITY, l = 0.f;
    int it = 0;
    bool ok = true;
    for (int j = 0; j < nt && ok; ++j) {
      if (!atc_tile_live(j, p, n0b, n1b)) continue;
      const int st = it & 1;
      const bool got = __all_sync(0xffffffffu, mbar_wait(&s_full[st], (it >> 1) & 1, abort_flag, p.err, kErrWaitAccFull));
      if (!got) {
        ok = false;
        break;
      }
      tc_fence_after();
      // the whole S row of this thread: four TMEM reads in flight, one wait
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) tmem_ld32(trow + st * BKV + c * 32, sr[c]);
      tmem_wait_ld();
      // valid keys of this tile form a prefix [0, nv)
      const int nv = j < p.nt0 ? min(BKV, min(n0b, p.L0) - j * BKV) : min(BKV, min(n1b, p.L1) - (j - p.nt0) * BKV);
      float s[BKV];
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < BKV; ++c) {
        s[c] = c < nv ? __uint_as_float(sr[c >> 5][c & 31]) * p.scale_log2 : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      const float mn = fmaxf(m, mt);
      const float corr = ex2_ftz(m - mn);  // 0 on the first tile (m = -inf)
      float ps = 0.f;
#pragma unroll
      for (int c = 0; c < BKV; ++c) {
        s[c] = ex2_ftz(s[c] - mn);
        ps += s[c];
      }
      l = l * corr + ps;
      m = mn;
      // O (TMEM) and the P buffer are free once the previous P V product has completed
      if (it >= 1) {
        const bool done = __all_sync(0xffffffffu, mbar_wait(o_done, (it - 1) & 1, abort_flag, p.err, kErrWaitAccFull));
        if (!done) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t r[16];
          tmem_ld16(trow + O_COL + c * 16, r);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 16; ++k) r[k] = __float_as_uint(__uint_as_float(r[k]) * corr);
          tmem_st16(trow + O_COL + c * 16, r);
        }
        tmem_wait_st();
      }
      // P_j: row `row` of a [128 x 128] bf16 K-major tile, two 64-key atoms with the 128-byte swizzle
      uint8_t* pb = sP + st * P_BYTES;
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const int c0 = a * 64 + ch * 8;
          uint4 w;
          w.x = pack_bf16(s[c0 + 0], s[c0 + 1]);
          w.y = pack_bf16(s[c0 + 2], s[c0 + 3]);
          w.z = pack_bf16(s[c0 + 4], s[c0 + 5]);
          w.w = pack_bf16(s[c0 + 6], s[c0 + 7]);
          *reinterpret_cast<uint4*>(pb + a * (P_BYTES / 2) + row * 128 + ((ch ^ (row & 7)) << 4)) = w;
        }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
      ++it;
    }
    // epilogue: O / l and the log-sum-exp (natural log)
    if (ok && it > 0) {
      const bool done = __all_sync(0xffffffffu, mbar_wait(o_done, (it - 1) & 1, abort_flag, p.err, kErrWaitAccFull));
      if (done) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const int qrow = q0 + row;
        float o[D];
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + O_COL + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[c * 32 + k] = __uint_as_float(r[k]) * inv;
        }
        if (qrow < p.Lq) {
          uint4* dst = reinterpret_cast<uint4*>(p.o + ((int64_t)b * p.Lq + qrow) * p.ldo + h * D);
#pragma unroll
          for (int k = 0; k < D / 8; ++k) {
            uint4 w;
            w.x = pack_bf16(o[8 * k + 0], o[8 * k + 1]);
            w.y = pack_bf16(o[8 * k + 2], o[8 * k + 3]);
            w.z = pack_bf16(o[8 * k + 4], o[8 * k + 5]);
            w.w = pack_bf16(o[8 * k + 6], o[8 * k + 7]);
            dst[k] = w;
          }
          p.lse[((int64_t)b * p.H + h) * p.Lq + qrow] = (m + log2f(l)) * kLn2;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ==================================================================================== forward, two query tiles
// Persistent; work item = (sample, head, 256 queries). Two softmax warpgroups each own one 128-query tile (A, B) and
// share every K/V tile the TMA warp loads. The MMA warp ping-pongs between them, so the tensor core works on one tile
// while the other's softmax runs:
//     S_A(0) S_B(0) | PV_A(0) S_A(1) | PV_B(0) S_B(1) | PV_A(1) S_A(2) | ...
// Q (two tiles) and K/V are double-buffered across items. TMEM: S_A [0,128), S_B [128,256), O_A [256,320),
// O_B [320,384).
namespace at2 {
constexpr int BQ = 128, BKV = 128, D = 64;
constexpr int THREADS = 320;                 // warp 0 TMA, warp 1 MMA, warps 2..5 softmax A, 6..9 softmax B
constexpr int QT = BQ * D * 2;               // 16 KiB: one Q tile
constexpr int KVT = BKV * D * 2;             // 16 KiB: one K or V tile
constexpr int PT = BQ * BKV * 2;             // 32 KiB: one P tile
constexpr int OFF_Q = 0;                     // [2 buffers][A, B]
constexpr int OFF_KV = OFF_Q + 4 * QT;       // [2 stages][K, V]
constexpr int OFF_P = OFF_KV + 4 * KVT;      // [A, B]
constexpr int OFF_BAR = OFF_P + 2 * PT;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t C_S = 0, C_O = 256;       // + X * 128 (S), + X * 64 (O)
}  // namespace at2

struct AttnTc2Params {
  const int *n0, *n1;
  int Lq, L0, L1, H;
  int nt0, nt1, nqp, items;
  float scale_log2;
  bf16* o;
  int64_t ldo;
  float* lse;
  int* err;
};

__device__ __forceinline__ int at2_live_tiles(const AttnTc2Params& p, int n0b, int n1b) {
  int n = 0;
  for (int j = 0; j < p.nt0; ++j) n += (j * at2::BKV < n0b) ? 1 : 0;
  for (int j = 0; j < p.nt1; ++j) n += (j * at2::BKV < n1b) ? 1 : 0;
  return n;
}

// j-th live key tile of a sample -> storage tile index (source 0 tiles first)
__device__ __forceinline__ int at2_tile(const AttnTc2Params& p, int n0b, int n1b, int live) {
  for (int j = 0; j < p.nt0; ++j)
    if (j * at2::BKV < n0b && live-- == 0) return j;
  for (int j = 0; j < p.nt1; ++j)
    if (j * at2::BKV < n1b && live-- == 0) return p.nt0 + j;
  return -1;
}

__global__ void __launch_bounds__(at2::THREADS)
    attn_fwd_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK0,
                        const __grid_constant__ CUtensorMap tmV0, const __grid_constant__ CUtensorMap tmK1,
                        const __grid_constant__ CUtensorMap tmV1, const AttnTc2Params p) {
  using namespace at2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;        // [2]
  uint64_t* q_empty = bars + 2;   // [2]
  uint64_t* kv_full = bars + 4;   // [2]
  uint64_t* kv_empty = bars + 6;  // [2]
  uint64_t* s_full = bars + 8;    // [A, B]
  uint64_t* p_full = bars + 10;   // [A, B]  (4 warps arrive)
  uint64_t* o_done = bars + 12;   // [A, B]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t g = 0;  // global live key-tile counter (K/V ring position)
      int ii = 0;
      for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x, ++ii) {
        const int bh = item / p.nqp, qp = item - bh * p.nqp, b = bh / p.H, h = bh - b * p.H;
        const int n0b = p.n0[b], n1b = p.n1[b];
        const int q0 = qp * 2 * BQ;
        const bool liveB = q0 + BQ < p.Lq;
        const int qb = ii & 1;
        if (!mbar_wait(&q_empty[qb], ((ii >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&q_full[qb], (liveB ? 2 : 1) * QT);
        tma_load_3d(&tmQ, &q_full[qb], smem + OFF_Q + (qb * 2) * QT, h * D, q0, b);
        if (liveB) tma_load_3d(&tmQ, &q_full[qb], smem + OFF_Q + (qb * 2 + 1) * QT, h * D, q0 + BQ, b);
        const int n = at2_live_tiles(p, n0b, n1b);
        for (int it = 0; it < n; ++it, ++g) {
          const int st = g & 1;
          if (!mbar_wait(&kv_empty[st], ((g >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
          const int j = at2_tile(p, n0b, n1b, it);
          uint8_t* k = smem + OFF_KV + st * 2 * KVT;
          mbar_arrive_expect_tx(&kv_full[st], 2 * KVT);
          if (j < p.nt0) {
            tma_load_3d(&tmK0, &kv_full[st], k, h * D, j * BKV, b);
            tma_load_3d(&tmV0, &kv_full[st], k + KVT, h * D, j * BKV, b);
          } else {
            tma_load_3d(&tmK1, &kv_full[st], k, h * D, (j - p.nt0) * BKV, b);
            tma_load_3d(&tmV1, &kv_full[st], k + KVT, h * D, (j - p.nt0) * BKV, b);
          }
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(BQ, BKV, 0, 0);
      constexpr uint32_t idesc_o = idesc_bf16_f32(BQ, D, 0, 1);
      uint32_t g = 0;   // K/V ring and tile-A barrier phases: every live key tile
      uint32_t gB = 0;  // tile-B barrier phases: key tiles of items whose tile B holds queries
      int ii = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x, ++ii) {
        const int bh = item / p.nqp, qp = item - bh * p.nqp, b = bh / p.H;
        const int n0b = p.n0[b], n1b = p.n1[b];
        const bool liveB = qp * 2 * BQ + BQ < p.Lq;
        const int qb = ii & 1;
        const int n = at2_live_tiles(p, n0b, n1b);
        if (!mbar_wait(&q_full[qb], (ii >> 1) & 1, abort_flag, p.err, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t qa = smem_u32(smem + OFF_Q + (qb * 2) * QT);
        auto issue_s = [&](int X, uint32_t gg) {
          const uint32_t kb = smem_u32(smem + OFF_KV + (gg & 1) * 2 * KVT);
          const uint32_t qx = qa + X * QT;
#pragma unroll
          for (int k = 0; k < D / 16; ++k)
            umma_f16(tmem + C_S + X * BKV, smem_desc_sw128(qx + k * 32, 16, 1024),
                     smem_desc_sw128(kb + k * 32, 16, 1024), idesc_s, k != 0 ? 1u : 0u);
          umma_commit(&s_full[X]);
        };
        auto issue_pv = [&](int X, uint32_t gg, bool first) {
          const uint32_t pa = smem_u32(smem + OFF_P + X * PT);
          const uint32_t vb = smem_u32(smem + OFF_KV + (gg & 1) * 2 * KVT + KVT);
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k)
            umma_f16(tmem + C_O + X * D, smem_desc_sw128(pa + (k >> 2) * (PT / 2) + (k & 3) * 32, 16, 1024),
                     smem_desc_sw128(vb + k * 2048, 8192, 1024), idesc_o, (!first || k != 0) ? 1u : 0u);
          umma_commit(&o_done[X]);
        };
        if (n > 0) {
          if (!mbar_wait(&kv_full[g & 1], (g >> 1) & 1, abort_flag, p.err, kErrWaitFull)) break;
          tc_fence_after();
          issue_s(0, g);
          if (liveB) issue_s(1, g);
        }
        for (int it = 0; it < n; ++it, ++g) {
          const bool more = it + 1 < n;
          if (!mbar_wait(&p_full[0], g & 1, abort_flag, p.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(0, g, it == 0);
          if (more) {
            if (!mbar_wait(&kv_full[(g + 1) & 1], ((g + 1) >> 1) & 1, abort_flag, p.err, kErrWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(0, g + 1);
          }
          if (liveB) {
            if (!mbar_wait(&p_full[1], gB & 1, abort_flag, p.err, kErrWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(1, g, it == 0);
            ++gB;
          }
          umma_commit(&kv_empty[g & 1]);
          if (more && liveB) issue_s(1, g + 1);
        }
        umma_commit(&q_empty[qb]);
      }
    }
  } else {
    // ---------------------------------------------------------------------------------------- softmax warpgroups
    const int X = (warp - 2) >> 2;  // 0: tile A, 1: tile B
    const int quarter = warp & 3;   // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    uint8_t* pb = smem + OFF_P + X * PT;
    uint32_t g = 0;  // this warpgroup's key tiles so far (its barriers' phases)
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x) {
      const int bh = item / p.nqp, qp = item - bh * p.nqp, b = bh / p.H, h = bh - b * p.H;
      const int n0b = p.n0[b], n1b = p.n1[b];
      const int q0 = qp * 2 * BQ + X * BQ;
      const int n = at2_live_tiles(p, n0b, n1b);
      if (q0 >= p.Lq) continue;  // tile B past the queries: the MMA warp skips it too
      float m = -INFINITY, l = 0.f;
      for (int it = 0; it < n; ++it, ++g) {
        const int j = at2_tile(p, n0b, n1b, it);
        const bool got = __all_sync(0xffffffffu, mbar_wait(&s_full[X], g & 1, abort_flag, p.err, kErrWaitAccFull));
        if (!got) {
          ok = false;
          break;
        }
        tc_fence_after();
        // valid keys of this tile: a prefix [0, nv)
        const int nv = j < p.nt0 ? min(BKV, min(n0b, p.L0) - j * BKV) : min(BKV, min(n1b, p.L1) - (j - p.nt0) * BKV);
        // pass 1: the row maximum, 32 columns at a time (TMEM reads are cheap; registers are not)
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < BKV / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + C_S + X * BKV + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (c * 32 + k < nv) mt = fmaxf(mt, __uint_as_float(r[k]));
        }
        const float mn = fmaxf(m, mt * p.scale_log2);
        const float corr = ex2_ftz(m - mn);
        m = mn;
        if (it >= 1) {
          // O and the P buffer are free once the previous P V product completed; S(g) was issued after PV(g-1), so
          // by now this wait returns at once
          const bool done =
              __all_sync(0xffffffffu, mbar_wait(&o_done[X], (g - 1) & 1, abort_flag, p.err, kErrWaitAccFull));
          if (!done) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (!__all_sync(0xffffffffu, corr == 1.f)) {
#pragma unroll
            for (int c = 0; c < D / 16; ++c) {
              uint32_t r[16];
              tmem_ld16(trow + C_O + X * D + c * 16, r);
              tmem_wait_ld();
#pragma unroll
              for (int k = 0; k < 16; ++k) r[k] = __float_as_uint(__uint_as_float(r[k]) * corr);
              tmem_st16(trow + C_O + X * D + c * 16, r);
            }
            tmem_wait_st();
          }
        }
        // pass 2: P = exp2(s * scale - max) straight into the shared-memory P tile (bf16, 128-byte swizzle: two
        // 64-key atoms); the row sum in fp32
        float ps = 0.f;
#pragma unroll
        for (int c = 0; c < BKV / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + C_S + X * BKV + c * 32, r);
          tmem_wait_ld();
          uint32_t w[16];
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float e0 = c * 32 + k < nv ? ex2_ftz(fmaf(__uint_as_float(r[k]), p.scale_log2, -mn)) : 0.f;
            const float e1 = c * 32 + k + 1 < nv ? ex2_ftz(fmaf(__uint_as_float(r[k + 1]), p.scale_log2, -mn)) : 0.f;
            ps += e0 + e1;
            w[k / 2] = pack_bf16(e0, e1);
          }
          // 32 keys = chunks 4 (c & 1) .. 4 (c & 1) + 3 of atom c / 2
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int ch = (c & 1) * 4 + q4;
            *reinterpret_cast<uint4*>(pb + (c >> 1) * (PT / 2) + row * 128 + ((ch ^ (row & 7)) << 4)) =
                make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]);
          }
        }
        l = l * corr + ps;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[X]);
      }
      if (!ok) break;
      // epilogue: O / l and the log-sum-exp (natural log); rows past Lq are not stored
      const int qrow = q0 + row;
      if (n > 0) {
        const bool done =
            __all_sync(0xffffffffu, mbar_wait(&o_done[X], (g - 1) & 1, abort_flag, p.err, kErrWaitAccFull));
        if (!done) break;
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(p.o + ((int64_t)b * p.Lq + min(qrow, p.Lq - 1)) * p.ldo + h * D);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + C_O + X * D + c * 32, r);
          tmem_wait_ld();
          if (qrow < p.Lq) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              dst[c * 4 + k] = make_uint4(pack_bf16(__uint_as_float(r[8 * k + 0]) * inv, __uint_as_float(r[8 * k + 1]) * inv),
                                          pack_bf16(__uint_as_float(r[8 * k + 2]) * inv, __uint_as_float(r[8 * k + 3]) * inv),
                                          pack_bf16(__uint_as_float(r[8 * k + 4]) * inv, __uint_as_float(r[8 * k + 5]) * inv),
                                          pack_bf16(__uint_as_float(r[8 * k + 6]) * inv, __uint_as_float(r[8 * k + 7]) * inv));
          }
        }
        tc_fence_before();
        if (qrow < p.Lq) p.lse[((int64_t)b * p.H + h) * p.Lq + qrow] = (m + log2f(l)) * atc::kLn2;
      } else if (qrow < p.Lq) {  // no valid key: zero output, lse = -inf (nothing to attend to)
        uint4* dst = reinterpret_cast<uint4*>(p.o + ((int64_t)b * p.Lq + qrow) * p.ldo + h * D);
#pragma unroll
        for (int k = 0; k < D / 8; ++k) dst[k] = make_uint4(0, 0, 0, 0);
        p.lse[((int64_t)b * p.H + h) * p.Lq + qrow] = -INFINITY;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ==================================================================================== forward, version 3 (default)
// Persistent; work item = (sample, head, 256 queries) with two softmax warpgroups (A, B), one 128-query tile each,
// sharing every K/V tile, as version 2. Three changes take the softmax off the tensor core's critical path:
//  * a softmax thread reads its whole S row (128 columns) into registers behind one wait and releases the S buffer
//    at once (s_free): S(j+1) = Q K(j+1)^T then runs on the tensor core while the exponentials of tile j are computed;
//  * P is double-buffered in shared memory per query tile, so P(j+1) is written while P(j) V(j) still runs. Q is
//    single-buffered to make room: the next item's Q is loaded once this item's last S products have completed;
//  * a row's running maximum moves only when a tile's maximum exceeds it by more than kRescaleLog2 (log2 units), so
//    P stays below 2^kRescaleLog2 and O in TMEM is rescaled only when some row of the warp moved (after the previous
//    P V product has completed). The result is unchanged: O and l are scaled by the same 2^-m, whatever m is.
// The softmax arithmetic is counted in instructions per score: full key tiles skip the mask predicates, maxima use
// the three-input max, and pairs of scores share one packed (f32x2) FMA and one packed add.
// MMA issue order per key tile j: S_A(j+1) S_B(j+1) | PV_A(j) PV_B(j). TMEM: S_A [0,128), S_B [128,256),
// O_A [256,320), O_B [320,384).
namespace at3 {
constexpr int BQ = 128, BKV = 128, D = 64;
constexpr int THREADS = 320;                 // warp 0 TMA, warp 1 MMA, warps 2..5 softmax A, 6..9 softmax B
constexpr int QT = BQ * D * 2;               // 16 KiB: one Q tile
constexpr int KVT = BKV * D * 2;             // 16 KiB: one K or V tile
constexpr int PT = BQ * BKV * 2;             // 32 KiB: one P tile
constexpr int OFF_Q = 0;                     // [A, B]
constexpr int OFF_KV = OFF_Q + 2 * QT;       // [2 stages][K, V]
constexpr int OFF_P = OFF_KV + 4 * KVT;      // [A, B][2 buffers]
constexpr int OFF_BAR = OFF_P + 4 * PT;      // 224 KiB
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t C_S = 0, C_O = 256;       // + X * 128 (S), + X * 64 (O)
constexpr float kRescaleLog2 = 8.f;
}  // namespace at3

__global__ void __launch_bounds__(at3::THREADS, 1)
    attn_fwd_tc3_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK0,
                        const __grid_constant__ CUtensorMap tmV0, const __grid_constant__ CUtensorMap tmK1,
                        const __grid_constant__ CUtensorMap tmV1, const AttnTc2Params p) {
  using namespace at3;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;        // Q of the item landed
  uint64_t* q_empty = bars + 1;   // the item's S products completed (Q may be overwritten)
  uint64_t* kv_full = bars + 2;   // [2]
  uint64_t* kv_empty = bars + 4;  // [2]
  uint64_t* s_full = bars + 6;    // [A, B] S product completed
  uint64_t* s_free = bars + 8;    // [A, B] S read into registers (4 warps arrive)
  uint64_t* p_full = bars + 10;   // [A, B] P written (4 warps arrive)
  uint64_t* p_empty = bars + 12;  // [A0, A1, B0, B1] the P V product of that buffer completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&p_empty[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t g = 0;  // live key tiles loaded so far (K/V ring position)
      int ii = 0;
      for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x, ++ii) {
        const int bh = item / p.nqp, qp = item - bh * p.nqp, b = bh / p.H, h = bh - b * p.H;
        const int n0b = p.n0[b], n1b = p.n1[b];
        const int q0 = qp * 2 * BQ;
        const bool liveB = q0 + BQ < p.Lq;
        if (!mbar_wait(q_empty, (ii & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(q_full, (liveB ? 2 : 1) * QT);
        tma_load_3d(&tmQ, q_full, smem + OFF_Q, h * D, q0, b);
        if (liveB) tma_load_3d(&tmQ, q_full, smem + OFF_Q + QT, h * D, q0 + BQ, b);
        const int n = at2_live_tiles(p, n0b, n1b);
        bool ok = true;
        for (int it = 0; it < n; ++it, ++g) {
          const int st = g & 1;
          if (!mbar_wait(&kv_empty[st], ((g >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const int j = at2_tile(p, n0b, n1b, it);
          uint8_t* k = smem + OFF_KV + st * 2 * KVT;
          mbar_arrive_expect_tx(&kv_full[st], 2 * KVT);
          if (j < p.nt0) {
            tma_load_3d(&tmK0, &kv_full[st], k, h * D, j * BKV, b);
            tma_load_3d(&tmV0, &kv_full[st], k + KVT, h * D, j * BKV, b);
          } else {
            tma_load_3d(&tmK1, &kv_full[st], k, h * D, (j - p.nt0) * BKV, b);
            tma_load_3d(&tmV1, &kv_full[st], k + KVT, h * D, (j - p.nt0) * BKV, b);
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(BQ, BKV, 0, 0);
      constexpr uint32_t idesc_o = idesc_bf16_f32(BQ, D, 0, 1);
      uint32_t g = 0;                 // K/V ring position
      uint32_t ns[2] = {0u, 0u};      // S products issued per query tile (s_free phases)
      uint32_t np[2] = {0u, 0u};      // P V products issued per query tile (p_full phases, P buffer)
      int ii = 0;
      bool ok = true;
      // S_X = Q_X K^T of ring slot gg, once the previous S_X has been read
      auto issue_s = [&](int X, uint32_t gg) -> bool {
        if (ns[X] > 0 && !mbar_wait(&s_free[X], (ns[X] - 1) & 1, abort_flag, p.err, kErrWaitAccEmpty)) return false;
        tc_fence_after();
        const uint32_t kb = smem_u32(smem + OFF_KV + (gg & 1) * 2 * KVT);
        const uint32_t qx = smem_u32(smem + OFF_Q + X * QT);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          umma_f16(tmem + C_S + X * BKV, smem_desc_sw128(qx + k * 32, 16, 1024), smem_desc_sw128(kb + k * 32, 16, 1024),
                   idesc_s, k != 0 ? 1u : 0u);
        umma_commit(&s_full[X]);
        ++ns[X];
        return true;
      };
      // O_X (+)= P_X V of ring slot gg, once P_X is written
      auto issue_pv = [&](int X, uint32_t gg, bool first) -> bool {
        if (!mbar_wait(&p_full[X], np[X] & 1, abort_flag, p.err, kErrWaitFull)) return false;
        tc_fence_after();
        const int pbuf = X * 2 + (np[X] & 1);
        const uint32_t pa = smem_u32(smem + OFF_P + pbuf * PT);
        const uint32_t vb = smem_u32(smem + OFF_KV + (gg & 1) * 2 * KVT + KVT);
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k)
          umma_f16(tmem + C_O + X * D, smem_desc_sw128(pa + (k >> 2) * (PT / 2) + (k & 3) * 32, 16, 1024),
                   smem_desc_sw128(vb + k * 2048, 8192, 1024), idesc_o, (!first || k != 0) ? 1u : 0u);
        umma_commit(&p_empty[pbuf]);
        ++np[X];
        return true;
      };
      for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x, ++ii) {
        const int bh = item / p.nqp, qp = item - bh * p.nqp, b = bh / p.H;
        const int n0b = p.n0[b], n1b = p.n1[b];
        const bool liveB = qp * 2 * BQ + BQ < p.Lq;
        const int n = at2_live_tiles(p, n0b, n1b);
        if (!mbar_wait(q_full, ii & 1, abort_flag, p.err, kErrWaitFull)) break;
        tc_fence_after();
        if (n > 0) {
          if (!mbar_wait(&kv_full[g & 1], (g >> 1) & 1, abort_flag, p.err, kErrWaitFull)) break;
          tc_fence_after();
          ok = issue_s(0, g) && (!liveB || issue_s(1, g));
        }
        for (int it = 0; ok && it < n; ++it, ++g) {
          if (it + 1 < n) {
            if (!mbar_wait(&kv_full[(g + 1) & 1], ((g + 1) >> 1) & 1, abort_flag, p.err, kErrWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            ok = issue_s(0, g + 1) && (!liveB || issue_s(1, g + 1));
            if (!ok) break;
          } else {
            umma_commit(q_empty);  // every S product of the item is issued: Q is free once they complete
          }
          ok = issue_pv(0, g, it == 0) && (!liveB || issue_pv(1, g, it == 0));
          if (!ok) break;
          umma_commit(&kv_empty[g & 1]);
        }
        if (ok && n == 0) umma_commit(q_empty);
      }
    }
  } else {
    // ---------------------------------------------------------------------------------------- softmax warpgroups
    const int X = (warp - 2) >> 2;  // 0: tile A, 1: tile B
    const int quarter = warp & 3;   // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    uint32_t g = 0;  // key tiles this warpgroup has processed (phases of s_full / p_full, P buffer)
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x) {
      const int bh = item / p.nqp, qp = item - bh * p.nqp, b = bh / p.H, h = bh - b * p.H;
      const int n0b = p.n0[b], n1b = p.n1[b];
      const int q0 = qp * 2 * BQ + X * BQ;
      const int n = at2_live_tiles(p, n0b, n1b);
      if (q0 >= p.Lq) continue;  // tile B past the queries: the MMA warp skips it too
      float m = -INFINITY, l = 0.f;
      for (int it = 0; it < n; ++it, ++g) {
        const int j = at2_tile(p, n0b, n1b, it);
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[X], g & 1, abort_flag, p.err, kErrWaitAccFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s[BKV / 32][32];
#pragma unroll
        for (int c = 0; c < BKV / 32; ++c) tmem_ld32(trow + C_S + X * BKV + c * 32, s[c]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[X]);  // the tensor core may compute the next S into this buffer
        // valid keys of this tile: a prefix [0, nv); a full tile (every image-key tile) takes the path without
        // per-element predicates. nv depends on the sample and the tile only, so the branch is uniform.
        const int nv = j < p.nt0 ? min(BKV, min(n0b, p.L0) - j * BKV) : min(BKV, min(n1b, p.L1) - (j - p.nt0) * BKV);
        const bool full = nv >= BKV;
        float mt;
        if (full) {  // two chains of three-input maxima
          float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
          for (int c = 0; c < BKV / 32; ++c)
#pragma unroll
            for (int k = 0; k < 32; k += 4) {
              ma = fmax3(ma, __uint_as_float(s[c][k]), __uint_as_float(s[c][k + 1]));
              mb = fmax3(mb, __uint_as_float(s[c][k + 2]), __uint_as_float(s[c][k + 3]));
            }
          mt = fmaxf(ma, mb);
        } else {
          mt = -INFINITY;
#pragma unroll
          for (int c = 0; c < BKV / 32; ++c)
#pragma unroll
            for (int k = 0; k < 32; ++k)
              if (c * 32 + k < nv) mt = fmaxf(mt, __uint_as_float(s[c][k]));
        }
        const float mn = mt * p.scale_log2;
        // the first tile sets the row maximum; later tiles move it only by more than kRescaleLog2
        const bool move = it > 0 && mn > m + kRescaleLog2;
        const float corr = move ? ex2_ftz(m - mn) : 1.f;
        if (it == 0 || move) m = mn;
        const bool rescale = __any_sync(0xffffffffu, move);
        // this tile's P buffer (g & 1) was last read by the P V product two tiles back
        if (g >= 2) {
          const uint32_t gp = g - 2;
          if (!__all_sync(0xffffffffu, mbar_wait(&p_empty[X * 2 + (gp & 1)], (gp >> 1) & 1, abort_flag, p.err,
                                                 kErrWaitAccFull))) {
            ok = false;
            break;
          }
        }
        // P = exp2(s * scale - m) (pairs: one packed FMA, two ex2, one packed add to the row sum, one bf16x2 pack)
        // into the shared-memory P tile (bf16, 128-byte swizzle: two 64-key atoms). Masked keys of a partial tile
        // get P = 0 (selected, so an overflowing exponential of an ignored key cannot leak).
        uint8_t* pb = smem + OFF_P + (X * 2 + (g & 1)) * PT;
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m, -m);
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < BKV / 32; ++c) {
          uint32_t w[16];
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float2 x = ffma2(make_float2(__uint_as_float(s[c][k]), __uint_as_float(s[c][k + 1])), sc2, nm2);
            float e0 = ex2_ftz(x.x), e1 = ex2_ftz(x.y);
            if (!full) {
              e0 = c * 32 + k < nv ? e0 : 0.f;
              e1 = c * 32 + k + 1 < nv ? e1 : 0.f;
            }
            acc = fadd2(acc, make_float2(e0, e1));
            w[k / 2] = pack_bf16(e0, e1);
          }
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int ch = (c & 1) * 4 + q4;
            *reinterpret_cast<uint4*>(pb + (c >> 1) * (PT / 2) + row * 128 + ((ch ^ (row & 7)) << 4)) =
                make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]);
          }
        }
        if (rescale) {
          // O holds P(0..it-1) V relative to the old maximum: rescale it, once the last P V product has completed,
          // before this tile's product (issued after p_full below) adds to it
          const uint32_t gp = g - 1;
          if (!__all_sync(0xffffffffu, mbar_wait(&p_empty[X * 2 + (gp & 1)], (gp >> 1) & 1, abort_flag, p.err,
                                                 kErrWaitAccFull))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 16; ++c) {
            uint32_t r[16];
            tmem_ld16(trow + C_O + X * D + c * 16, r);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 16; ++k) r[k] = __float_as_uint(__uint_as_float(r[k]) * corr);
            tmem_st16(trow + C_O + X * D + c * 16, r);
          }
          tmem_wait_st();
        }
        l = l * corr + (acc.x + acc.y);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[X]);
      }
      if (!ok) break;
      // epilogue: O / l and the log-sum-exp (natural log); rows past Lq are not stored
      const int qrow = q0 + row;
      if (n > 0) {
        const uint32_t gp = g - 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&p_empty[X * 2 + (gp & 1)], (gp >> 1) & 1, abort_flag, p.err,
                                               kErrWaitAccFull)))
          break;
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(p.o + ((int64_t)b * p.Lq + min(qrow, p.Lq - 1)) * p.ldo + h * D);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + C_O + X * D + c * 32, r);
          tmem_wait_ld();
          if (qrow < p.Lq) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              dst[c * 4 + k] = make_uint4(pack_bf16(__uint_as_float(r[8 * k + 0]) * inv, __uint_as_float(r[8 * k + 1]) * inv),
                                          pack_bf16(__uint_as_float(r[8 * k + 2]) * inv, __uint_as_float(r[8 * k + 3]) * inv),
                                          pack_bf16(__uint_as_float(r[8 * k + 4]) * inv, __uint_as_float(r[8 * k + 5]) * inv),
                                          pack_bf16(__uint_as_float(r[8 * k + 6]) * inv, __uint_as_float(r[8 * k + 7]) * inv));
          }
        }
        tc_fence_before();
        if (qrow < p.Lq) p.lse[((int64_t)b * p.H + h) * p.Lq + qrow] = (m + log2f(l)) * atc::kLn2;
      } else if (qrow < p.Lq) {  // no valid key: zero output, lse = -inf (nothing to attend to)
        uint4* dst = reinterpret_cast<uint4*>(p.o + ((int64_t)b * p.Lq + qrow) * p.ldo + h * D);
#pragma unroll
        for (int k = 0; k < D / 8; ++k) dst[k] = make_uint4(0, 0, 0, 0);
        p.lse[((int64_t)b * p.H + h) * p.Lq + qrow] = -INFINITY;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ====================================================================================================== torch glue
// Cycle counters for the profiled instantiations (kBwdProf* slots of the backward), or null: set by attn_prof_set
// with a device uint64 tensor of at least 16 entries (a diagnostic; the normal instantiations record nothing).
static unsigned long long* g_attn_prof = nullptr;  // at least 20 counters

void attn_prof_set(const c10::optional<at::Tensor>& counters) {
  if (counters.has_value() && counters->defined()) {
    TORCH_CHECK(counters->is_cuda() && counters->scalar_type() == at::kLong && counters->numel() >= 20,
                "attn_prof_set: a CUDA int64 tensor of at least 20 counters");
    g_attn_prof = reinterpret_cast<unsigned long long*>(counters->data_ptr());
  } else {
    g_attn_prof = nullptr;
  }
}

// 3-D map over a token-major view [B * L rows, C] with row stride ld: dims (C, L, B), box (64, 128, 1).
static CUtensorMap seq_map(const at::Tensor& t, int64_t L) {
  const int64_t B = t.size(0) / L;
  return make_tmap_bf16(t.data_ptr(), t.size(1), L, B, t.stride(0), t.stride(0) * L, atc::D, atc::BKV);
}

void attn_fwd_tc(const at::Tensor& q, const at::Tensor& k0, const at::Tensor& v0, const c10::optional<at::Tensor>& k1,
                 const c10::optional<at::Tensor>& v1, const at::Tensor& n0, const at::Tensor& n1, const at::Tensor& o,
                 const at::Tensor& lse, int64_t Lq, int64_t L0, int64_t L1, double scale, int64_t version) {
  TORCH_CHECK(q.is_cuda() && q.size(1) % 64 == 0, "attn_fwd_tc: head dim 64");
  TORCH_CHECK(n0.scalar_type() == at::kInt && n1.scalar_type() == at::kInt, "int32 key counts expected");
  const at::cuda::CUDAGuard guard(q.device());
  const bool has1 = k1.has_value() && k1->defined() && L1 > 0;
  AttnTcParams p{};
  p.n0 = n0.data_ptr<int>();
  p.n1 = n1.data_ptr<int>();
  p.Lq = (int)Lq;
  p.L0 = (int)L0;
  p.L1 = has1 ? (int)L1 : 0;
  p.H = (int)(q.size(1) / 64);
  p.nt0 = (int)((L0 + atc::BKV - 1) / atc::BKV);
  p.nt1 = has1 ? (int)((L1 + atc::BKV - 1) / atc::BKV) : 0;
  p.scale_log2 = (float)scale * atc::kLog2e;
  p.o = reinterpret_cast<bf16*>(o.data_ptr());
  p.ldo = o.stride(0);
  p.lse = lse.data_ptr<float>();
  p.err = status_word();
  CUtensorMap mq = make_tmap_bf16(q.data_ptr(), q.size(1), Lq, q.size(0) / Lq, q.stride(0), q.stride(0) * Lq, atc::D,
                                  atc::BQ);
  CUtensorMap mk0 = seq_map(k0, L0), mv0 = seq_map(v0, L0);
  CUtensorMap mk1 = has1 ? seq_map(*k1, L1) : mk0, mv1 = has1 ? seq_map(*v1, L1) : mv0;
  const int B = (int)(q.size(0) / Lq);
  if (version == 1) {
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, atc::SMEM);
      attr = true;
    }
    dim3 grid((unsigned)((Lq + atc::BQ - 1) / atc::BQ), (unsigned)(B * p.H));
    attn_fwd_tc_kernel<<<grid, atc::THREADS, atc::SMEM, at::cuda::getCurrentCUDAStream()>>>(mq, mk0, mv0, mk1, mv1,
                                                                                             p);
    NG_LAUNCH_CHECK();
    return;
  }
  AttnTc2Params p2{};
  p2.n0 = p.n0;
  p2.n1 = p.n1;
  p2.Lq = p.Lq;
  p2.L0 = p.L0;
  p2.L1 = p.L1;
  p2.H = p.H;
  p2.nt0 = p.nt0;
  p2.nt1 = p.nt1;
  p2.nqp = (int)((Lq + 2 * at2::BQ - 1) / (2 * at2::BQ));
  p2.items = B * p.H * p2.nqp;
  p2.scale_log2 = p.scale_log2;
  p2.o = p.o;
  p2.ldo = p.ldo;
  p2.lse = p.lse;
  p2.err = p.err;
  static bool attr2 = false;
  static int sms = 0;
  if (!attr2) {
    cudaFuncSetAttribute(attn_fwd_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, at2::SMEM);
    cudaFuncSetAttribute(attn_fwd_tc3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, at3::SMEM);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, q.get_device());
    attr2 = true;
  }
  const int grid = std::max(1, std::min(p2.items, sms));
  if (version == 2)
    attn_fwd_tc2_kernel<<<grid, at2::THREADS, at2::SMEM, at::cuda::getCurrentCUDAStream()>>>(mq, mk0, mv0, mk1, mv1,
                                                                                             p2);
  else
    attn_fwd_tc3_kernel<<<grid, at3::THREADS, at3::SMEM, at::cuda::getCurrentCUDAStream()>>>(mq, mk0, mv0, mk1, mv1,
                                                                                             p2);
  NG_LAUNCH_CHECK();
}


// ====================================================================================================== backward
// One CTA per (128-key tile, sample, head); loops over 128-query tiles i:
//   MMA warp       S^T  = K Q_i^T, dP^T = V dO_i^T          (M = 128 keys, N = 128 queries, K = 64) into TMEM
//   compute warps  (a thread per key row) P^T = exp(S^T * scale - lse), dS^T = P^T (dP^T - delta), both bf16 into
//                  shared memory (K-major over queries: two 64-query swizzle atoms)
//   MMA warp       dV += P^T dO_i, dK += dS^T Q_i           (M = 128 keys, N = 64, K = 128 queries; dO_i, Q_i as
//                                                            MN-major operands)
//                  dQ_i = dS K                               (M = 128 queries: dS^T read as an MN-major A operand)
//   compute warps  (a thread per query row) scale * dQ_i -> fp32 tiles -> TMA reduce-add into an fp32 dQ buffer
// dV and dK stay in TMEM across the query tiles and are written once (keys without validity get zeros).
namespace atb {
constexpr int BQ = 128, BK = 128, D = 64;
constexpr int THREADS = 192;
constexpr int T16 = BK * D * 2;        // 16 KiB: a [128 x 64] bf16 tile
constexpr int PT = BK * BQ * 2;        // 32 KiB: P^T or dS^T [128 keys x 128 queries]
constexpr int OFF_K = 0, OFF_V = T16, OFF_Q = 2 * T16, OFF_DO = 4 * T16, OFF_P = 6 * T16, OFF_DS = OFF_P + PT;
constexpr int OFF_DQ = OFF_DS + PT;    // per compute warp: 2 x [32 rows x 32 fp32] = 8 KiB; 4 warps = 32 KiB
constexpr int OFF_LSE = OFF_DQ + 32768;
constexpr int SMEM = OFF_LSE + 4 * 2 * BQ * 4 + 1024 + 256;  // + per compute warp lse/delta, barriers
constexpr uint32_t TMEM_COLS = 512;    // S^T [0,128), dP^T [128,256), dV [256,320), dK [320,384), dQ [384,448)
constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 320, C_DQ = 384;
}  // namespace atb

struct AttnTcBwdParams {
  const int *n0, *n1;
  int Lq, L0, L1, H;
  int nt0, nt1, nq;
  float scale, scale_log2;
  const float* lse;
  const float* delta;
  bf16 *dk0, *dv0, *dk1, *dv1;
  int64_t lddk0, lddv0, lddk1, lddv1;
  int* err;
};

__global__ void __launch_bounds__(atb::THREADS, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmK0, const __grid_constant__ CUtensorMap tmV0,
                       const __grid_constant__ CUtensorMap tmK1, const __grid_constant__ CUtensorMap tmV1,
                       const __grid_constant__ CUtensorMap tmDQ, const AttnTcBwdParams p) {
  using namespace atb;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sLse = reinterpret_cast<float*>(smem + OFF_LSE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_LSE + 4 * 2 * BQ * 4);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;   // [2]
  uint64_t* qd_empty = bars + 3;  // [2]
  uint64_t* st_full = bars + 5;
  uint64_t* ps_full = bars + 6;
  uint64_t* dq_full = bars + 7;
  uint64_t* dq_empty = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int n0b = p.n0[b], n1b = p.n1 ? p.n1[b] : 0;
  const bool src1 = j >= p.nt0;
  const int kt0 = (src1 ? j - p.nt0 : j) * BK;  // first row of this tile in its source
  const int Lsrc = src1 ? p.L1 : p.L0;
  const int nvalid = src1 ? n1b : n0b;
  const bool live = kt0 < nvalid && kt0 < Lsrc;

  bf16* dk_base = src1 ? p.dk1 : p.dk0;
  bf16* dv_base = src1 ? p.dv1 : p.dv0;
  const int64_t lddk = src1 ? p.lddk1 : p.lddk0, lddv = src1 ? p.lddv1 : p.lddv0;

  if (!live) {
    // no valid key in this tile: zero gradients for its existing rows
    for (int idx = threadIdx.x; idx < BK * 8; idx += blockDim.x) {
      const int r = idx >> 3, ch = idx & 7;
      const int s = kt0 + r;
      if (s >= Lsrc) continue;
      const int64_t row = (int64_t)b * Lsrc + s;
      *reinterpret_cast<uint4*>(dk_base + row * lddk + h * D + ch * 8) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(dv_base + row * lddv + h * D + ch * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(ps_full, 4);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // --------------------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * T16);
      tma_load_3d(src1 ? &tmK1 : &tmK0, kv_full, smem + OFF_K, h * D, kt0, b);
      tma_load_3d(src1 ? &tmV1 : &tmV0, kv_full, smem + OFF_V, h * D, kt0, b);
      for (int i = 0; i < p.nq; ++i) {
        const int st = i & 1;
        if (!mbar_wait(&qd_empty[st], ((i >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&qd_full[st], 2 * T16);
        tma_load_3d(&tmQ, &qd_full[st], smem + OFF_Q + st * T16, h * D, i * BQ, b);
        tma_load_3d(&tmDO, &qd_full[st], smem + OFF_DO + st * T16, h * D, i * BQ, b);
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(BK, BQ, 0, 0);  // M keys, N queries, both K-major over d
      constexpr uint32_t id_kv = idesc_bf16_f32(BK, D, 0, 1);  // M keys, N = d (MN-major), K = queries
      constexpr uint32_t id_q = idesc_bf16_f32(BQ, D, 1, 1);   // M queries (dS^T as MN-major A), N = d, K = keys
      const uint32_t aK = smem_u32(smem + OFF_K), aV = smem_u32(smem + OFF_V);
      const uint32_t aP = smem_u32(smem + OFF_P), aDS = smem_u32(smem + OFF_DS);
      bool ok = mbar_wait(kv_full, 0, abort_flag, p.err, kErrWaitFull);
      for (int i = 0; ok && i < p.nq; ++i) {
        const int st = i & 1;
        if (!mbar_wait(&qd_full[st], (i >> 1) & 1, abort_flag, p.err, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t aQ = smem_u32(smem + OFF_Q + st * T16), aDO = smem_u32(smem + OFF_DO + st * T16);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          umma_f16(tmem + C_S, smem_desc_sw128(aK + k * 32, 16, 1024), smem_desc_sw128(aQ + k * 32, 16, 1024), id_s,
                   k != 0 ? 1u : 0u);
          umma_f16(tmem + C_DP, smem_desc_sw128(aV + k * 32, 16, 1024), smem_desc_sw128(aDO + k * 32, 16, 1024),
                   id_s, k != 0 ? 1u : 0u);
        }
        umma_commit(st_full);
        if (!mbar_wait(ps_full, i & 1, abort_flag, p.err, kErrWaitFull)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k) {
          const uint32_t ka = (k >> 2) * (PT / 2) + (k & 3) * 32;  // K-major over queries: atom, then 32 B steps
          umma_f16(tmem + C_DV, smem_desc_sw128(aP + ka, 16, 1024), smem_desc_sw128(aDO + k * 2048, 8192, 1024),
                   id_kv, (i != 0 || k != 0) ? 1u : 0u);
          umma_f16(tmem + C_DK, smem_desc_sw128(aDS + ka, 16, 1024), smem_desc_sw128(aQ + k * 2048, 8192, 1024),
                   id_kv, (i != 0 || k != 0) ? 1u : 0u);
        }
        if (i >= 1 && !mbar_wait(dq_empty, (i - 1) & 1, abort_flag, p.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)  // A = dS (queries x keys): dS^T rows are keys -> MN-major, 16 keys per step
          umma_f16(tmem + C_DQ, smem_desc_sw128(aDS + k * 2048, PT / 2, 1024),
                   smem_desc_sw128(aK + k * 2048, 8192, 1024), id_q, k != 0 ? 1u : 0u);
        umma_commit(dq_full);
        umma_commit(&qd_empty[st]);
      }
    }
  } else {
    // --------------------------------------------------------------------------------------- compute warps
    const int qq = warp & 3;
    const int r = qq * 32 + lane;                        // key row (P/dS phase) or query row (dQ phase)
    const uint32_t trow = tmem + ((uint32_t)(qq * 32) << 16);
    const bool key_ok = (kt0 + r) < nvalid && (kt0 + r) < Lsrc;
    uint8_t* dq_st = smem + OFF_DQ + (warp - 2) * 8192;  // this warp's two [32 x 32] fp32 tiles
    const float* lse_bh = p.lse + ((int64_t)b * p.H + h) * p.Lq;
    const float* del_bh = p.delta + ((int64_t)b * p.H + h) * p.Lq;
    float* wLse = sLse + (warp - 2) * 2 * BQ;  // this warp's copy of the query tile's lse (log2 units) and delta
    float* wDel = wLse + BQ;
    bool ok = true;
    for (int i = 0; i < p.nq && ok; ++i) {
      __syncwarp();
#pragma unroll
      for (int k = 0; k < BQ / 32; ++k) {
        const int qg = i * BQ + k * 32 + lane;
        wLse[k * 32 + lane] = qg < p.Lq ? lse_bh[qg] * atc::kLog2e : INFINITY;
        wDel[k * 32 + lane] = qg < p.Lq ? del_bh[qg] : 0.f;
      }
      __syncwarp();
      const bool got = __all_sync(0xffffffffu, mbar_wait(st_full, i & 1, abort_flag, p.err, kErrWaitAccFull));
      if (!got) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint8_t* sP = smem + OFF_P;
      uint8_t* sDS = smem + OFF_DS;
#pragma unroll 1
      for (int c = 0; c < BQ / 32; ++c) {
        uint32_t rs[32], rd[32];
        tmem_ld32(trow + C_S + c * 32, rs);
        tmem_ld32(trow + C_DP + c * 32, rd);
        tmem_wait_ld();
        float pv[32], dv[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int qc = c * 32 + k;
          const float pk = key_ok ? exp2f(__uint_as_float(rs[k]) * p.scale_log2 - wLse[qc]) : 0.f;
          pv[k] = pk;
          dv[k] = pk * (__uint_as_float(rd[k]) - wDel[qc]);
        }
        // 32 queries = half of a 64-query atom: atom c / 2, chunks 4 * (c % 2) .. +3
        const int atom = c >> 1;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          const int cc = (c & 1) * 4 + ch;
          const uint32_t off = atom * (PT / 2) + r * 128 + ((cc ^ (r & 7)) << 4);
          uint4 w;
          w.x = pack_bf16(pv[8 * ch + 0], pv[8 * ch + 1]);
          w.y = pack_bf16(pv[8 * ch + 2], pv[8 * ch + 3]);
          w.z = pack_bf16(pv[8 * ch + 4], pv[8 * ch + 5]);
          w.w = pack_bf16(pv[8 * ch + 6], pv[8 * ch + 7]);
          *reinterpret_cast<uint4*>(sP + off) = w;
          w.x = pack_bf16(dv[8 * ch + 0], dv[8 * ch + 1]);
          w.y = pack_bf16(dv[8 * ch + 2], dv[8 * ch + 3]);
          w.z = pack_bf16(dv[8 * ch + 4], dv[8 * ch + 5]);
          w.w = pack_bf16(dv[8 * ch + 6], dv[8 * ch + 7]);
          *reinterpret_cast<uint4*>(sDS + off) = w;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ps_full);
      // dQ_i: rows are queries now
      const bool dq = __all_sync(0xffffffffu, mbar_wait(dq_full, i & 1, abort_flag, p.err, kErrWaitAccFull));
      if (!dq) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) bulk_wait_read0();  // the previous tile's dQ stores have read the staging tiles
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t rq[32];
        tmem_ld32(trow + C_DQ + c * 32, rq);
        tmem_wait_ld();
        uint8_t* t = dq_st + c * 4096;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)
          *reinterpret_cast<float4*>(t + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(rq[4 * ch]) * p.scale, __uint_as_float(rq[4 * ch + 1]) * p.scale,
                          __uint_as_float(rq[4 * ch + 2]) * p.scale, __uint_as_float(rq[4 * ch + 3]) * p.scale);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(dq_empty);
        tma_reduce_add_3d(&tmDQ, dq_st, h * D, i * BQ + qq * 32, b);
        tma_reduce_add_3d(&tmDQ, dq_st + 4096, h * D + 32, i * BQ + qq * 32, b);
        bulk_commit();
      }
    }
    // dV, dK (complete once the last dq_full arrived: their MMAs were committed before it). The TMEM loads are
    // warp-collective (.sync.aligned): every lane issues them; only the stores depend on the row existing.
    if (ok) {
      tc_fence_after();
      const int s = kt0 + r;
      const int64_t row = (int64_t)b * Lsrc + s;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        float v[D];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t rr[32];
          tmem_ld32(trow + (which ? C_DK : C_DV) + c * 32, rr);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) v[c * 32 + k] = __uint_as_float(rr[k]) * (which ? p.scale : 1.f);
        }
        if (s < Lsrc) {
          bf16* dst = which ? dk_base + row * lddk + h * D : dv_base + row * lddv + h * D;
#pragma unroll
          for (int k = 0; k < D / 8; ++k) {
            uint4 w;
            w.x = pack_bf16(v[8 * k + 0], v[8 * k + 1]);
            w.y = pack_bf16(v[8 * k + 2], v[8 * k + 3]);
            w.z = pack_bf16(v[8 * k + 4], v[8 * k + 5]);
            w.w = pack_bf16(v[8 * k + 6], v[8 * k + 7]);
            reinterpret_cast<uint4*>(dst)[k] = w;
          }
        }
      }
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ================================================================================ backward, persistent version
// Work item = (128-key tile, sample, head); a CTA loops over items with K/V double-buffered, so the next item's loads
// and S^T/dP^T MMAs overlap this item's dK/dV epilogue. Eight compute warps: two per TMEM lane quarter, warp half h
// owns query columns [64h, 64h + 64) of S^T/dP^T (= one 64-query swizzle atom of P^T/dS^T), d columns
// [32h, 32h + 32) of dQ, dK, dV. dQ tiles are staged for their TMA reduce-add in the warp's own 4 KiB slice of the
// P^T tile, which the dV MMA has finished reading when dQ is ready.
// TMEM: S^T [0,128), dP^T [128,256), dV [256,320), dK [320,384), dQ [384,448).
namespace ab2 {
constexpr int BQ = 128, BK = 128, D = 64;
constexpr int THREADS = 320;                       // warp 0 TMA, warp 1 MMA, warps 2..9 compute
constexpr int T16 = BK * D * 2;                    // 16 KiB
constexpr int PT = BK * BQ * 2;                    // 32 KiB
constexpr int OFF_KV = 0;                          // [2 buffers][K, V]
constexpr int OFF_QD = OFF_KV + 4 * T16;           // [2 stages][Q, dO]
constexpr int OFF_P = OFF_QD + 4 * T16;            // P^T
constexpr int OFF_DS = OFF_P + PT;                 // dS^T
constexpr int OFF_LD = OFF_DS + PT;                // [2 stages][128 queries] float2 (lse in log2 units, delta)
constexpr int OFF_BAR = OFF_LD + 2 * BQ * 8;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 320, C_DQ = 384;
}  // namespace ab2

struct AttnTcBwd2Params {
  const int *n0, *n1;
  int Lq, L0, L1, H;
  int nt0, nt1, nq, items;
  float scale, scale_log2;
  const float2* ld;  // [B, H, nq * 128] (lse * log2(e), delta); rows past Lq hold (+inf, 0)
  bf16 *dk0, *dv0, *dk1, *dv1;
  int64_t lddk0, lddv0, lddk1, lddv1;
  int* err;
};

struct Bwd2Item {
  int b, h, kt0, Lsrc, nvalid;
  bool src1, live;
};

__device__ __forceinline__ Bwd2Item bwd2_item(const AttnTcBwd2Params& p, int item) {
  Bwd2Item it;
  const int nt = p.nt0 + p.nt1;
  const int j = item % nt, bh = item / nt;
  it.b = bh / p.H;
  it.h = bh - it.b * p.H;
  it.src1 = j >= p.nt0;
  it.kt0 = (it.src1 ? j - p.nt0 : j) * ab2::BK;
  it.Lsrc = it.src1 ? p.L1 : p.L0;
  it.nvalid = it.src1 ? p.n1[it.b] : p.n0[it.b];
  it.live = it.kt0 < it.nvalid && it.kt0 < it.Lsrc;
  return it;
}

__global__ void __launch_bounds__(ab2::THREADS)
    attn_bwd_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                        const __grid_constant__ CUtensorMap tmK0, const __grid_constant__ CUtensorMap tmV0,
                        const __grid_constant__ CUtensorMap tmK1, const __grid_constant__ CUtensorMap tmV1,
                        const __grid_constant__ CUtensorMap tmDQ, const AttnTcBwd2Params p) {
  using namespace ab2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars;         // [2]
  uint64_t* kv_empty = bars + 2;    // [2]
  uint64_t* qd_full = bars + 4;     // [2]
  uint64_t* qd_empty = bars + 6;    // [2]
  uint64_t* st_full = bars + 8;
  uint64_t* ps_full = bars + 9;     // 8 warps
  uint64_t* dq_full = bars + 10;
  uint64_t* dq_empty = bars + 11;   // 8 warps
  uint64_t* dkv_full = bars + 12;
  uint64_t* dkv_empty = bars + 13;  // 8 warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(ps_full, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 8);
    mbar_init(dkv_full, 1);
    mbar_init(dkv_empty, 8);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t li = 0, gq = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x) {
        const Bwd2Item w = bwd2_item(p, item);
        if (!w.live) continue;
        const int kb = li & 1;
        if (!mbar_wait(&kv_empty[kb], ((li >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&kv_full[kb], 2 * T16);
        tma_load_3d(w.src1 ? &tmK1 : &tmK0, &kv_full[kb], smem + OFF_KV + kb * 2 * T16, w.h * D, w.kt0, w.b);
        tma_load_3d(w.src1 ? &tmV1 : &tmV0, &kv_full[kb], smem + OFF_KV + kb * 2 * T16 + T16, w.h * D, w.kt0, w.b);
        for (int i = 0; i < p.nq; ++i, ++gq) {
          const int st = gq & 1;
          if (!mbar_wait(&qd_empty[st], ((gq >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&qd_full[st], 2 * T16 + BQ * 8);
          tma_load_3d(&tmQ, &qd_full[st], smem + OFF_QD + st * 2 * T16, w.h * D, i * BQ, w.b);
          tma_load_3d(&tmDO, &qd_full[st], smem + OFF_QD + st * 2 * T16 + T16, w.h * D, i * BQ, w.b);
          bulk_load(smem + OFF_LD + st * BQ * 8, p.ld + ((int64_t)w.b * p.H + w.h) * p.nq * BQ + i * BQ, BQ * 8,
                    &qd_full[st]);
        }
        ++li;
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(BK, BQ, 0, 0);
      constexpr uint32_t id_kv = idesc_bf16_f32(BK, D, 0, 1);
      constexpr uint32_t id_q = idesc_bf16_f32(BQ, D, 1, 1);
      const uint32_t aP = smem_u32(smem + OFF_P), aDS = smem_u32(smem + OFF_DS);
      uint32_t li = 0, gq = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x) {
        const Bwd2Item w = bwd2_item(p, item);
        if (!w.live) continue;
        const int kb = li & 1;
        if (!mbar_wait(&kv_full[kb], (li >> 1) & 1, abort_flag, p.err, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t aK = smem_u32(smem + OFF_KV + kb * 2 * T16), aV = aK + T16;
        for (int i = 0; i < p.nq; ++i, ++gq) {
          const int st = gq & 1;
          if (!mbar_wait(&qd_full[st], (gq >> 1) & 1, abort_flag, p.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aQ = smem_u32(smem + OFF_QD + st * 2 * T16), aDO = aQ + T16;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            umma_f16(tmem + C_S, smem_desc_sw128(aK + k * 32, 16, 1024), smem_desc_sw128(aQ + k * 32, 16, 1024), id_s,
                     k != 0 ? 1u : 0u);
            umma_f16(tmem + C_DP, smem_desc_sw128(aV + k * 32, 16, 1024), smem_desc_sw128(aDO + k * 32, 16, 1024),
                     id_s, k != 0 ? 1u : 0u);
          }
          umma_commit(st_full);
          if (!mbar_wait(ps_full, gq & 1, abort_flag, p.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          if (i == 0 && li >= 1 && !mbar_wait(dkv_empty, (li - 1) & 1, abort_flag, p.err, kErrWaitAccEmpty)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < BQ / 16; ++k) {
            const uint32_t ka = (k >> 2) * (PT / 2) + (k & 3) * 32;
            umma_f16(tmem + C_DV, smem_desc_sw128(aP + ka, 16, 1024), smem_desc_sw128(aDO + k * 2048, 8192, 1024),
                     id_kv, (i != 0 || k != 0) ? 1u : 0u);
            umma_f16(tmem + C_DK, smem_desc_sw128(aDS + ka, 16, 1024), smem_desc_sw128(aQ + k * 2048, 8192, 1024),
                     id_kv, (i != 0 || k != 0) ? 1u : 0u);
          }
          if (gq >= 1 && !mbar_wait(dq_empty, (gq - 1) & 1, abort_flag, p.err, kErrWaitAccEmpty)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(tmem + C_DQ, smem_desc_sw128(aDS + k * 2048, PT / 2, 1024),
                     smem_desc_sw128(aK + k * 2048, 8192, 1024), id_q, k != 0 ? 1u : 0u);
          umma_commit(dq_full);
          umma_commit(&qd_empty[st]);
        }
        if (!ok) break;
        umma_commit(dkv_full);
        umma_commit(&kv_empty[kb]);
        ++li;
      }
    }
  } else {
    // ------------------------------------------------------------------------------------------ compute warps
    const int quarter = warp & 3, hh = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // key row (P/dS, dK/dV) or query row (dQ) of this thread
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const float2* lds = reinterpret_cast<const float2*>(smem + OFF_LD);   // [2 stages][128]
    uint8_t* slice = smem + OFF_P + hh * (PT / 2) + quarter * 4096;        // this warp's 4 KiB of P^T
    uint32_t li = 0, gq = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x) {
      const Bwd2Item w = bwd2_item(p, item);
      bf16* dk_base = w.src1 ? p.dk1 : p.dk0;
      bf16* dv_base = w.src1 ? p.dv1 : p.dv0;
      const int64_t lddk = w.src1 ? p.lddk1 : p.lddk0, lddv = w.src1 ? p.lddv1 : p.lddv0;
      const int s_row = w.kt0 + r;
      const int64_t grow = (int64_t)w.b * w.Lsrc + min(s_row, w.Lsrc - 1);
      if (!w.live) {  // no valid key in the tile: zero gradients for its rows
        if (s_row < w.Lsrc) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            reinterpret_cast<uint4*>(dk_base + grow * lddk + w.h * D + hh * 32)[k] = make_uint4(0, 0, 0, 0);
            reinterpret_cast<uint4*>(dv_base + grow * lddv + w.h * D + hh * 32)[k] = make_uint4(0, 0, 0, 0);
          }
        }
        continue;
      }
      const bool key_ok = s_row < w.nvalid && s_row < w.Lsrc;
      for (int i = 0; i < p.nq; ++i, ++gq) {
        const float2* ldq = lds + (gq & 1) * BQ + hh * 64;  // this warp's 64 queries: (lse log2, delta)
        if (lane == 0) bulk_wait_read0();  // the previous dQ tile staged in this slice has been read
        __syncwarp();
        if (!__all_sync(0xffffffffu, mbar_wait(st_full, gq & 1, abort_flag, p.err, kErrWaitAccFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          // S^T and dP^T of 32 queries: both TMEM reads in flight, one wait (all four would exceed the registers)
          uint32_t rs[1][32], rd[1][32];
          tmem_ld32(trow + C_S + hh * 64 + c * 32, rs[0]);
          tmem_ld32(trow + C_DP + hh * 64 + c * 32, rd[0]);
          tmem_wait_ld();
          // 32 queries = 16-byte chunks 4c .. 4c + 3 of the warp's 64-query atom, 8 queries per chunk
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint32_t wp[4], wd[4];
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
              const int kk = q4 * 8 + k;
              const float2 a0 = ldq[c * 32 + kk], a1 = ldq[c * 32 + kk + 1];
              const float p0 = key_ok ? ex2_ftz(fmaf(__uint_as_float(rs[0][kk]), p.scale_log2, -a0.x)) : 0.f;
              const float p1 = key_ok ? ex2_ftz(fmaf(__uint_as_float(rs[0][kk + 1]), p.scale_log2, -a1.x)) : 0.f;
              wp[k / 2] = pack_bf16(p0, p1);
              wd[k / 2] = pack_bf16(p0 * (__uint_as_float(rd[0][kk]) - a0.y),
                                    p1 * (__uint_as_float(rd[0][kk + 1]) - a1.y));
            }
            const int ch = c * 4 + q4;
            const uint32_t off = hh * (PT / 2) + r * 128 + ((ch ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(smem + OFF_P + off) = make_uint4(wp[0], wp[1], wp[2], wp[3]);
            *reinterpret_cast<uint4*>(smem + OFF_DS + off) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ps_full);
        // dQ_i (rows are queries now): scale, stage in this warp's P^T slice, reduce-add by TMA
        if (!__all_sync(0xffffffffu, mbar_wait(dq_full, gq & 1, abort_flag, p.err, kErrWaitAccFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        {
          uint32_t rq[32];
          tmem_ld32(trow + C_DQ + hh * 32, rq);
          tmem_wait_ld();
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            *reinterpret_cast<float4*>(slice + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
                make_float4(__uint_as_float(rq[4 * ch]) * p.scale, __uint_as_float(rq[4 * ch + 1]) * p.scale,
                            __uint_as_float(rq[4 * ch + 2]) * p.scale, __uint_as_float(rq[4 * ch + 3]) * p.scale);
        }
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(dq_empty);
          tma_reduce_add_3d(&tmDQ, slice, w.h * D + hh * 32, i * BQ + quarter * 32, w.b);
          bulk_commit();
        }
      }
      if (!ok) break;
      // dV, dK of the item: 32 d columns of this warp half, key rows of its quarter
      if (!__all_sync(0xffffffffu, mbar_wait(dkv_full, li & 1, abort_flag, p.err, kErrWaitAccFull))) break;
      tc_fence_after();
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        uint32_t rr[32];
        tmem_ld32(trow + (which ? C_DK : C_DV) + hh * 32, rr);
        tmem_wait_ld();
        if (s_row < w.Lsrc) {
          const float sc = which ? p.scale : 1.f;
          uint4* dst = reinterpret_cast<uint4*>((which ? dk_base + grow * lddk : dv_base + grow * lddv) + w.h * D +
                                                hh * 32);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            dst[k] = make_uint4(pack_bf16(__uint_as_float(rr[8 * k]) * sc, __uint_as_float(rr[8 * k + 1]) * sc),
                                pack_bf16(__uint_as_float(rr[8 * k + 2]) * sc, __uint_as_float(rr[8 * k + 3]) * sc),
                                pack_bf16(__uint_as_float(rr[8 * k + 4]) * sc, __uint_as_float(rr[8 * k + 5]) * sc),
                                pack_bf16(__uint_as_float(rr[8 * k + 6]) * sc, __uint_as_float(rr[8 * k + 7]) * sc));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dkv_empty);
      ++li;
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ================================================================================ backward, version 3 (default)
// Persistent; work item = (sample, head): every key tile j of the sample and its (at most two) 128-query tiles i, so
// dQ_i accumulates in TMEM over the key tiles and is written once as bf16 (no fp32 buffer, no reduce-adds, no store
// pass), while dK_j / dV_j accumulate over the query tiles. Per (j, i), in issue order:
//   MMA      S^T = K_j Q_i^T, dP^T = V_j dO_i^T  (M = 128 keys, N = 128 queries)                 -> st_full
//   compute  S^T and dP^T rows into registers -> s_free: the MMA warp issues the next (j, i)'s S^T and dP^T; this
//            thread forms P^T = exp2(S^T scale log2(e) - lse_i) and dS^T = P^T (dP^T - delta_i) in registers while
//            the previous (j, i)'s products run, and overwrites the P^T / dS^T tiles (bf16, 128-byte swizzle) once
//            those have completed (mma_done)                                                     -> ps_full
//   MMA      dV_j += P^T dO_i, dK_j += dS^T Q_i, dQ_i += dS K_j                                    -> mma_done
// After the last i of a key tile the compute warps read dK_j and dV_j (dkv_full) and store them (dkv_empty); after
// the last key tile they read dQ_0, dQ_1 (dq_full) and store them (dq_empty). Key tiles without a valid key are not
// loaded; their dK / dV rows are written as zeros. The next item's Q / dO are loaded once this item's products have
// completed (single buffer). Sixteen compute warps, four per TMEM lane quarter: warp w of a quarter takes query
// columns [32 w, 32 w + 32) of S^T / dP^T (so a thread holds 64 values, not 128, and twice the warps hide the
// latencies), d columns [16 w, 16 w + 16) of dK / dV, and query tile w / 2, d columns [32 (w % 2), +32) of dQ.
// Samples with more than two query tiles take version 2.
// TMEM: S^T [0,128), dP^T [128,256), dV [256,320), dK [320,384), dQ_0 [384,448), dQ_1 [448,512).
namespace ab3 {
constexpr int BQ = 128, BK = 128, D = 64;
constexpr int THREADS = 576;                 // warp 0 TMA, warp 1 MMA, warps 2..17 compute
constexpr int NCW = 16;                      // compute warps
constexpr int T16 = BK * D * 2;              // 16 KiB: one [128 x 64] bf16 tile
constexpr int PT = BK * BQ * 2;              // 32 KiB: P^T or dS^T [128 keys x 128 queries]
constexpr int MAXQ = 2;                      // query tiles per item
constexpr int OFF_QD = 0;                    // [Q_0, Q_1, dO_0, dO_1]
constexpr int OFF_KV = OFF_QD + 4 * T16;     // [2 stages][K, V]
constexpr int OFF_P = OFF_KV + 4 * T16;      // P^T
constexpr int OFF_DS = OFF_P + PT;           // dS^T
constexpr int OFF_LD = OFF_DS + PT;          // [MAXQ][128] float2 (lse in log2 units, delta)
constexpr int OFF_BAR = OFF_LD + MAXQ * BQ * 8;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 320, C_DQ = 384;  // dQ_i at C_DQ + 64 i
}  // namespace ab3

struct AttnTcBwd3Params {
  const int *n0, *n1;
  int Lq, L0, L1, H;
  int nt0, nt1, nq, items;
  float scale, scale_log2;
  const float2* ld;  // [B, H, nq * 128] (lse * log2(e), delta); rows past Lq hold (+inf, 0)
  bf16 *dq, *dk0, *dv0, *dk1, *dv1;
  int64_t lddq, lddk0, lddv0, lddk1, lddv1;
  int* err;
  unsigned long long* prof;  // cycle counters of the profiled instantiation (kBwdProf* slots), else null
};

// Cycle counters of the profiled backward (per CTA, summed over the warps of a role; see attn_prof_set):
enum : int {
  kBwdProfWaitSt = 0, kBwdProfExp, kBwdProfWaitMma, kBwdProfStore, kBwdProfWaitDkv, kBwdProfEpiDkv, kBwdProfWaitDq,
  kBwdProfEpiDq, kBwdProfCompute, kBwdProfMmaWaitQd, kBwdProfMmaWaitKv, kBwdProfMmaWaitSfree, kBwdProfMmaWaitPs,
  kBwdProfMmaWaitEpi, kBwdProfMma, kBwdProfTmaWait, kBwdProfWaitQd, kBwdProfItem, kBwdProfMmaIssueS,
  kBwdProfMmaIssueProd, kBwdProfSlots
};

struct Bwd3Tile {
  int kt0, Lsrc, nvalid;
  bool src1, live;
};

__device__ __forceinline__ Bwd3Tile bwd3_tile(const AttnTcBwd3Params& p, int b, int j) {
  Bwd3Tile t;
  t.src1 = j >= p.nt0;
  t.kt0 = (t.src1 ? j - p.nt0 : j) * ab3::BK;
  t.Lsrc = t.src1 ? p.L1 : p.L0;
  t.nvalid = min(t.src1 ? p.n1[b] : p.n0[b], t.Lsrc);
  t.live = t.kt0 < t.nvalid;
  return t;
}

template <bool PROF>
__global__ void __launch_bounds__(ab3::THREADS, 1)
    attn_bwd_tc3_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                        const __grid_constant__ CUtensorMap tmK0, const __grid_constant__ CUtensorMap tmV0,
                        const __grid_constant__ CUtensorMap tmK1, const __grid_constant__ CUtensorMap tmV1,
                        const AttnTcBwd3Params p) {
  using namespace ab3;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* qd_full = bars;          // Q, dO and the lse / delta rows of the item landed
  uint64_t* qd_empty = bars + 1;     // the item's products completed
  uint64_t* kv_full = bars + 2;      // [2]
  uint64_t* kv_empty = bars + 4;     // [2]
  uint64_t* st_full = bars + 6;      // S^T and dP^T computed
  uint64_t* s_free = bars + 7;       // S^T and dP^T read (compute warps)
  uint64_t* ps_full = bars + 8;      // P^T and dS^T written (compute warps)
  uint64_t* mma_done = bars + 9;     // the products of the last (j, i) completed
  uint64_t* dkv_full = bars + 10;    // dK_j, dV_j complete
  uint64_t* dkv_empty = bars + 11;   // dK_j, dV_j read (compute warps)
  uint64_t* dq_full = bars + 12;     // dQ of the item complete
  uint64_t* dq_empty = bars + 13;    // dQ read (compute warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int nt = p.nt0 + p.nt1;
  __shared__ unsigned long long prof_s[kBwdProfSlots];
#define NG_PROF_T0(v) const uint64_t v = PROF ? clock64() : 0
#define NG_PROF_ADD(k, v) \
  if (PROF && lane == 0) atomicAdd(&prof_s[k], (unsigned long long)(clock64() - v))

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (PROF && threadIdx.x < kBwdProfSlots) prof_s[threadIdx.x] = 0;
  if (threadIdx.x == 0) {
    mbar_init(qd_full, 1);
    mbar_init(qd_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(s_free, NCW);
    mbar_init(ps_full, NCW);
    mbar_init(mma_done, 1);
    mbar_init(dkv_full, 1);
    mbar_init(dkv_empty, NCW);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, NCW);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t li = 0;  // live key tiles loaded so far (K/V ring position)
      int ii = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x, ++ii) {
        const int b = item / p.H, h = item - b * p.H;
        NG_PROF_T0(tq);
        if (!mbar_wait(qd_empty, (ii & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
        NG_PROF_ADD(kBwdProfTmaWait, tq);
        mbar_arrive_expect_tx(qd_full, p.nq * (2 * T16 + BQ * 8));
        for (int i = 0; i < p.nq; ++i) {
          tma_load_3d(&tmQ, qd_full, smem + OFF_QD + i * T16, h * D, i * BQ, b);
          tma_load_3d(&tmDO, qd_full, smem + OFF_QD + (2 + i) * T16, h * D, i * BQ, b);
        }
        bulk_load(smem + OFF_LD, p.ld + ((int64_t)b * p.H + h) * p.nq * BQ, p.nq * BQ * 8, qd_full);
        for (int j = 0; j < nt; ++j) {
          const Bwd3Tile t = bwd3_tile(p, b, j);
          if (!t.live) continue;
          const int st = li & 1;
          NG_PROF_T0(tk);
          if (!mbar_wait(&kv_empty[st], ((li >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          NG_PROF_ADD(kBwdProfTmaWait, tk);
          mbar_arrive_expect_tx(&kv_full[st], 2 * T16);
          uint8_t* kv = smem + OFF_KV + st * 2 * T16;
          tma_load_3d(t.src1 ? &tmK1 : &tmK0, &kv_full[st], kv, h * D, t.kt0, b);
          tma_load_3d(t.src1 ? &tmV1 : &tmV0, &kv_full[st], kv + T16, h * D, t.kt0, b);
          ++li;
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      NG_PROF_T0(tmma);
      constexpr uint32_t id_s = idesc_bf16_f32(BK, BQ, 0, 0);
      constexpr uint32_t id_kv = idesc_bf16_f32(BK, D, 0, 1);
      constexpr uint32_t id_q = idesc_bf16_f32(BQ, D, 1, 1);
      const uint32_t aP = smem_u32(smem + OFF_P), aDS = smem_u32(smem + OFF_DS);
      uint32_t li = 0, gq = 0, nkt = 0, ndq = 0;
      int ii = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x, ++ii) {
        const int b = item / p.H;
        int nlive = 0;
        for (int j = 0; j < nt; ++j) nlive += bwd3_tile(p, b, j).live ? 1 : 0;
        NG_PROF_T0(tq);
        if (!mbar_wait(qd_full, ii & 1, abort_flag, p.err, kErrWaitFull)) break;
        NG_PROF_ADD(kBwdProfMmaWaitQd, tq);
        tc_fence_after();
        if (nlive == 0) {
          umma_commit(qd_empty);
          continue;
        }
        const int nq = p.nq, N = nlive * nq;
        auto issue_s = [&](int it) -> bool {
          const int t = it / nq, i = it - t * nq;
          const uint32_t slot = li + t;
          NG_PROF_T0(tk);
          if (i == 0 && !mbar_wait(&kv_full[slot & 1], (slot >> 1) & 1, abort_flag, p.err, kErrWaitFull)) return false;
          NG_PROF_ADD(kBwdProfMmaWaitKv, tk);
          const uint32_t g = gq + it;
          NG_PROF_T0(ts);
          if (g > 0 && !mbar_wait(s_free, (g - 1) & 1, abort_flag, p.err, kErrWaitAccEmpty)) return false;
          NG_PROF_ADD(kBwdProfMmaWaitSfree, ts);
          NG_PROF_T0(tis);
          tc_fence_after();
          const uint32_t aK = smem_u32(smem + OFF_KV + (slot & 1) * 2 * T16), aV = aK + T16;
          const uint32_t aQ = smem_u32(smem + OFF_QD + i * T16), aDO = smem_u32(smem + OFF_QD + (2 + i) * T16);
          // descriptors as base + (byte offset >> 4): the start-address field is the low 14 bits and shared memory is
          // below 2^18 bytes, so the add never carries out of it
          const uint64_t dK = smem_desc_sw128(aK, 16, 1024), dQ = smem_desc_sw128(aQ, 16, 1024);
          const uint64_t dV = smem_desc_sw128(aV, 16, 1024), dO = smem_desc_sw128(aDO, 16, 1024);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            umma_f16(tmem + C_S, dK + k * 2, dQ + k * 2, id_s, k != 0 ? 1u : 0u);
            umma_f16(tmem + C_DP, dV + k * 2, dO + k * 2, id_s, k != 0 ? 1u : 0u);
          }
          umma_commit(st_full);
          NG_PROF_ADD(kBwdProfMmaIssueS, tis);
          return true;
        };
        auto issue_prod = [&](int it) -> bool {
          const int t = it / nq, i = it - t * nq;
          const uint32_t slot = li + t;
          const uint32_t g = gq + it;
          NG_PROF_T0(tp);
          if (!mbar_wait(ps_full, g & 1, abort_flag, p.err, kErrWaitFull)) return false;
          NG_PROF_ADD(kBwdProfMmaWaitPs, tp);
          NG_PROF_T0(te);
          // dK / dV of the previous key tile read out before this tile's first products overwrite them
          if (i == 0 && nkt + t > 0 && !mbar_wait(dkv_empty, (nkt + t - 1) & 1, abort_flag, p.err, kErrWaitAccEmpty))
            return false;
          // dQ of the previous item read out before this item's first dQ products overwrite it
          if (it == 0 && ndq > 0 && !mbar_wait(dq_empty, (ndq - 1) & 1, abort_flag, p.err, kErrWaitAccEmpty))
            return false;
          NG_PROF_ADD(kBwdProfMmaWaitEpi, te);
          NG_PROF_T0(tip);
          tc_fence_after();
          const uint32_t aK = smem_u32(smem + OFF_KV + (slot & 1) * 2 * T16);
          const uint32_t aQ = smem_u32(smem + OFF_QD + i * T16), aDO = smem_u32(smem + OFF_QD + (2 + i) * T16);
          const uint64_t dP = smem_desc_sw128(aP, 16, 1024), dS = smem_desc_sw128(aDS, 16, 1024);
          const uint64_t dO = smem_desc_sw128(aDO, 8192, 1024), dQ = smem_desc_sw128(aQ, 8192, 1024);
#pragma unroll
          for (int k = 0; k < BQ / 16; ++k) {
            const uint32_t ka = ((k >> 2) * (PT / 2) + (k & 3) * 32) >> 4;
            umma_f16(tmem + C_DV, dP + ka, dO + k * 128, id_kv, (i != 0 || k != 0) ? 1u : 0u);
            umma_f16(tmem + C_DK, dS + ka, dQ + k * 128, id_kv, (i != 0 || k != 0) ? 1u : 0u);
          }
          const uint64_t dSm = smem_desc_sw128(aDS, PT / 2, 1024), dKm = smem_desc_sw128(aK, 8192, 1024);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(tmem + C_DQ + i * D, dSm + k * 128, dKm + k * 128, id_q, (t != 0 || k != 0) ? 1u : 0u);
          umma_commit(mma_done);
          if (i == nq - 1) {
            umma_commit(dkv_full);
            umma_commit(&kv_empty[slot & 1]);
          }
          NG_PROF_ADD(kBwdProfMmaIssueProd, tip);
          return true;
        };
        ok = issue_s(0);
        for (int it = 0; ok && it < N; ++it) {
          if (it + 1 < N) ok = issue_s(it + 1);
          ok = ok && issue_prod(it);
        }
        if (!ok) break;
        umma_commit(dq_full);
        umma_commit(qd_empty);
        gq += N;
        li += nlive;
        nkt += nlive;
        ++ndq;
      }
      NG_PROF_ADD(kBwdProfMma, tmma);
    }
  } else {
    // ------------------------------------------------------------------------------------------ compute warps
    const int quarter = warp & 3, cg = (warp - 2) >> 2;  // TMEM lane quarter; column group 0..3
    const int r = quarter * 32 + lane;  // key row (S^T, dP^T, dK, dV) or query row (dQ) of this thread
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    uint32_t gq = 0, nkt = 0, ndq = 0;
    int ii = 0;
    bool ok = true;
    // dK / dV of a key tile that is not the item's last live tile are read in the next live tile's first iteration,
    // after its exponentials (the wait for the tile's last products then overlaps them): the destination rows of the
    // pending tile, or null
    bf16 *pend_dk = nullptr, *pend_dv = nullptr;
    bool pend = false;
    // reads dK / dV of the finished key tile (once its last products completed), frees them, stores them
    auto flush_dkv = [&](bf16* dk_row, bf16* dv_row) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(dkv_full, nkt & 1, abort_flag, p.err, kErrWaitAccFull))) return false;
      tc_fence_after();
      uint32_t rv[16], rk[16];
      tmem_ld16(trow + C_DV + cg * 16, rv);
      tmem_ld16(trow + C_DK + cg * 16, rk);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dkv_empty);
      ++nkt;
      if (dk_row != nullptr) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          reinterpret_cast<uint4*>(dv_row)[k] =
              make_uint4(pack_bf16(__uint_as_float(rv[8 * k]), __uint_as_float(rv[8 * k + 1])),
                         pack_bf16(__uint_as_float(rv[8 * k + 2]), __uint_as_float(rv[8 * k + 3])),
                         pack_bf16(__uint_as_float(rv[8 * k + 4]), __uint_as_float(rv[8 * k + 5])),
                         pack_bf16(__uint_as_float(rv[8 * k + 6]), __uint_as_float(rv[8 * k + 7])));
          reinterpret_cast<uint4*>(dk_row)[k] =
              make_uint4(pack_bf16(__uint_as_float(rk[8 * k]) * p.scale, __uint_as_float(rk[8 * k + 1]) * p.scale),
                         pack_bf16(__uint_as_float(rk[8 * k + 2]) * p.scale, __uint_as_float(rk[8 * k + 3]) * p.scale),
                         pack_bf16(__uint_as_float(rk[8 * k + 4]) * p.scale, __uint_as_float(rk[8 * k + 5]) * p.scale),
                         pack_bf16(__uint_as_float(rk[8 * k + 6]) * p.scale, __uint_as_float(rk[8 * k + 7]) * p.scale));
        }
      }
      return true;
    };
    NG_PROF_T0(tall);
    for (int item = blockIdx.x; ok && item < p.items && !*abort_flag; item += gridDim.x, ++ii) {
      const int b = item / p.H, h = item - b * p.H;
      NG_PROF_T0(ti);
      int nlive = 0, last_live = -1;
      for (int j = 0; j < nt; ++j)
        if (bwd3_tile(p, b, j).live) {
          ++nlive;
          last_live = j;
        }
      NG_PROF_ADD(kBwdProfItem, ti);
      NG_PROF_T0(tqd);
      if (nlive > 0 && !__all_sync(0xffffffffu, mbar_wait(qd_full, ii & 1, abort_flag, p.err, kErrWaitFull))) break;
      NG_PROF_ADD(kBwdProfWaitQd, tqd);
      for (int j = 0; ok && j < nt; ++j) {
        const Bwd3Tile t = bwd3_tile(p, b, j);
        const int s_row = t.kt0 + r;
        // this thread's 16 columns of its key row in dK and dV
        auto dkv_rows = [&](bf16*& dk_row, bf16*& dv_row) {
          const int64_t grow = (int64_t)b * t.Lsrc + min(s_row, t.Lsrc - 1);
          dk_row = (t.src1 ? p.dk1 : p.dk0) + grow * (t.src1 ? p.lddk1 : p.lddk0) + h * D + cg * 16;
          dv_row = (t.src1 ? p.dv1 : p.dv0) + grow * (t.src1 ? p.lddv1 : p.lddv0) + h * D + cg * 16;
        };
        if (!t.live) {  // no valid key in the tile: zero gradients for its rows
          if (s_row < t.Lsrc) {
            bf16 *dk_row, *dv_row;
            dkv_rows(dk_row, dv_row);
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              reinterpret_cast<uint4*>(dk_row)[k] = make_uint4(0, 0, 0, 0);
              reinterpret_cast<uint4*>(dv_row)[k] = make_uint4(0, 0, 0, 0);
            }
          }
          continue;
        }
        const bool key_ok = s_row < t.nvalid;
        const bool all_ok = __all_sync(0xffffffffu, key_ok);
        for (int i = 0; i < p.nq; ++i, ++gq) {
          // (lse log2, delta) of this warp's 32 queries
          const float4* ld4 = reinterpret_cast<const float4*>(smem + OFF_LD) + (i * BQ + cg * 32) / 2;
          NG_PROF_T0(t0);
          if (!__all_sync(0xffffffffu, mbar_wait(st_full, gq & 1, abort_flag, p.err, kErrWaitAccFull))) {
            ok = false;
            break;
          }
          NG_PROF_ADD(kBwdProfWaitSt, t0);
          NG_PROF_T0(t1);
          tc_fence_after();
          // P^T and dS^T of these 32 queries, packed to bf16 pairs in registers, in two rounds of 16 (16-column TMEM
          // loads keep the registers below the cap of 18 warps); S^T / dP^T are released once the second round is in
          // registers. The exponentials run while the previous (j, i)'s products still read the P^T / dS^T tiles;
          // the tiles are overwritten once those have completed (mma_done). Per pair of queries: one 16-byte load of
          // both (lse, delta), one packed FMA, two ex2, one packed subtract, one packed multiply. Rows of keys past
          // the valid ones get zeros (selected); a warp whose keys are all valid skips the selects.
          uint32_t wp[16], wd[16];
          const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
#pragma unroll
          for (int h16 = 0; h16 < 2; ++h16) {
            uint32_t rs[16], rd[16];
            tmem_ld16(trow + C_S + cg * 32 + h16 * 16, rs);
            tmem_ld16(trow + C_DP + cg * 32 + h16 * 16, rd);
            tmem_wait_ld();
            if (h16 == 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(s_free);  // the next S^T / dP^T may be computed into these columns
            }
#pragma unroll
            for (int k = 0; k < 16; k += 2) {
              const float4 a = ld4[(h16 * 16 + k) >> 1];  // (lse0, delta0, lse1, delta1)
              const float2 x = ffma2(make_float2(__uint_as_float(rs[k]), __uint_as_float(rs[k + 1])), sc2,
                                     make_float2(-a.x, -a.z));
              float2 pr = make_float2(ex2_ftz(x.x), ex2_ftz(x.y));
              const float2 dd = fadd2(make_float2(__uint_as_float(rd[k]), __uint_as_float(rd[k + 1])),
                                      make_float2(-a.y, -a.w));
              float2 ds = fmul2(pr, dd);
              if (!all_ok) {
                pr = key_ok ? pr : make_float2(0.f, 0.f);
                ds = key_ok ? ds : make_float2(0.f, 0.f);
              }
              wp[(h16 * 16 + k) / 2] = pack_bf16(pr.x, pr.y);
              wd[(h16 * 16 + k) / 2] = pack_bf16(ds.x, ds.y);
            }
          }
          NG_PROF_ADD(kBwdProfExp, t1);
          NG_PROF_T0(t2);
          if (gq > 0 &&
              !__all_sync(0xffffffffu, mbar_wait(mma_done, (gq - 1) & 1, abort_flag, p.err, kErrWaitAccFull))) {
            ok = false;
            break;
          }
          NG_PROF_ADD(kBwdProfWaitMma, t2);
          NG_PROF_T0(t3);
          // 32 queries = 16-byte chunks 4 (cg & 1) .. + 3 of the 64-query swizzle atom cg / 2
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int ch = (cg & 1) * 4 + q4;
            const uint32_t off = (cg >> 1) * (PT / 2) + r * 128 + ((ch ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(smem + OFF_P + off) = make_uint4(wp[4 * q4], wp[4 * q4 + 1], wp[4 * q4 + 2],
                                                                       wp[4 * q4 + 3]);
            *reinterpret_cast<uint4*>(smem + OFF_DS + off) = make_uint4(wd[4 * q4], wd[4 * q4 + 1], wd[4 * q4 + 2],
                                                                        wd[4 * q4 + 3]);
          }
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(ps_full);
          NG_PROF_ADD(kBwdProfStore, t3);
          if (pend) {  // the previous key tile's dK / dV (its products completed before mma_done above)
            NG_PROF_T0(t5);
            pend = false;
            if (!flush_dkv(pend_dk, pend_dv)) {
              ok = false;
              break;
            }
            NG_PROF_ADD(kBwdProfEpiDkv, t5);
          }
        }
        if (!ok) break;
        // dV, dK of key tile j (16 d columns of this column group, key rows of its quarter): now for the item's last
        // live tile, else in the next live tile's first iteration
        bf16 *dk_row = nullptr, *dv_row = nullptr;
        if (s_row < t.Lsrc) dkv_rows(dk_row, dv_row);
        if (j != last_live) {
          pend = true;
          pend_dk = dk_row;
          pend_dv = dv_row;
          continue;
        }
        NG_PROF_T0(t4);
        if (!flush_dkv(dk_row, dv_row)) {
          ok = false;
          break;
        }
        NG_PROF_ADD(kBwdProfWaitDkv, t4);
      }
      if (!ok) break;
      // dQ of the item: column group cg takes query tile cg / 2, d columns [32 (cg % 2), +32), query rows of its
      // quarter
      const int qt = cg >> 1, dc = (cg & 1) * 32;
      const int qrow = qt * BQ + r;
      bf16* dq_row = p.dq + ((int64_t)b * p.Lq + min(qrow, p.Lq - 1)) * p.lddq + h * D + dc;
      if (nlive == 0) {  // nothing to attend to: zero gradients
        if (qt < p.nq && qrow < p.Lq)
#pragma unroll
          for (int k = 0; k < 4; ++k) reinterpret_cast<uint4*>(dq_row)[k] = make_uint4(0, 0, 0, 0);
        continue;
      }
      NG_PROF_T0(t6);
      if (!__all_sync(0xffffffffu, mbar_wait(dq_full, ndq & 1, abort_flag, p.err, kErrWaitAccFull))) break;
      NG_PROF_ADD(kBwdProfWaitDq, t6);
      NG_PROF_T0(t7);
      tc_fence_after();
      if (qt < p.nq) {
        uint32_t rq[32];
        tmem_ld32(trow + C_DQ + qt * D + dc, rq);
        tmem_wait_ld();
        if (qrow < p.Lq) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            reinterpret_cast<uint4*>(dq_row)[k] =
                make_uint4(pack_bf16(__uint_as_float(rq[8 * k]) * p.scale, __uint_as_float(rq[8 * k + 1]) * p.scale),
                           pack_bf16(__uint_as_float(rq[8 * k + 2]) * p.scale, __uint_as_float(rq[8 * k + 3]) * p.scale),
                           pack_bf16(__uint_as_float(rq[8 * k + 4]) * p.scale, __uint_as_float(rq[8 * k + 5]) * p.scale),
                           pack_bf16(__uint_as_float(rq[8 * k + 6]) * p.scale, __uint_as_float(rq[8 * k + 7]) * p.scale));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_empty);
      NG_PROF_ADD(kBwdProfEpiDq, t7);
      ++ndq;
    }
    NG_PROF_ADD(kBwdProfCompute, tall);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (PROF && threadIdx.x < kBwdProfSlots) atomicAdd(p.prof + threadIdx.x, prof_s[threadIdx.x]);
#undef NG_PROF_T0
#undef NG_PROF_ADD
}

// dq_acc[row, c] (fp32, TMA reduce-add target) -> dq (bf16, strided view)
__global__ void dq_store_kernel(const float* __restrict__ acc, bf16* __restrict__ dq, int64_t lddq, int64_t rows,
                                int C) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n8 = rows * (C / 8);
  if (t >= n8) return;
  const int64_t row = t / (C / 8);
  const int c8 = (int)(t - row * (C / 8));
  const float4 a = reinterpret_cast<const float4*>(acc + row * C)[2 * c8];
  const float4 b = reinterpret_cast<const float4*>(acc + row * C)[2 * c8 + 1];
  uint4 w;
  w.x = pack_bf16(a.x, a.y);
  w.y = pack_bf16(a.z, a.w);
  w.z = pack_bf16(b.x, b.y);
  w.w = pack_bf16(b.z, b.w);
  *reinterpret_cast<uint4*>(dq + row * lddq + c8 * 8) = w;
}

void attn_delta(const bf16* dout, int64_t lddo, const bf16* o, int64_t ldo, float* delta, int rows, int Lq, int H,
                cudaStream_t s);

// ld[b, h, q] = (lse * log2(e), sum_d dO * O) for q < Lq; (+inf, 0) for Lq <= q < Lqp (padding rows then give P = 0).
// Eight lanes per (row, head): each lane reads one 16-byte vector of dO and of O, so a warp reads 512 contiguous bytes
// of a row (four heads) per load, and the eight partial dots meet in three shuffles. Threads past the B * Lq * H * 8
// lanes fill the padding rows q >= Lq.
__global__ void attn_ld8_kernel(const bf16* __restrict__ dout, int64_t lddo, const bf16* __restrict__ o, int64_t ldo,
                                const float* __restrict__ lse, float2* __restrict__ ld, int B, int H, int Lq, int Lqp) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t lanes = (int64_t)B * Lq * H * 8;
  // every lane of the warp reaches the shuffles (a warp may hold both dot lanes and padding or idle lanes; groups of
  // eight never mix, since `lanes` is a multiple of 8)
  const bool dot = t < lanes;
  const int64_t unit = t >> 3;
  const int e = (int)(t & 7);
  const int64_t row = dot ? unit / H : 0;  // b * Lq + q
  const int h = dot ? (int)(unit - row * H) : 0;
  float acc = 0.f;
  if (dot) {
    const uint4 x = reinterpret_cast<const uint4*>(dout + row * lddo + h * 64)[e];
    const uint4 y = reinterpret_cast<const uint4*>(o + row * ldo + h * 64)[e];
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int k = 0; k < 4; ++k)
      acc += __uint_as_float(xs[k] << 16) * __uint_as_float(ys[k] << 16) +
             __uint_as_float(xs[k] & 0xffff0000u) * __uint_as_float(ys[k] & 0xffff0000u);
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (dot) {
    if (e == 0) {
      const int b = (int)(row / Lq), q = (int)(row - (int64_t)b * Lq);
      const int64_t bh = (int64_t)b * H + h;
      ld[bh * Lqp + q] = make_float2(lse[bh * Lq + q] * atc::kLog2e, acc);
    }
    return;
  }
  const int64_t u = t - lanes;  // padding rows
  const int pad = Lqp - Lq;
  if (pad <= 0 || u >= (int64_t)B * H * pad) return;
  const int64_t bh = u / pad;
  ld[bh * Lqp + Lq + (int)(u - bh * pad)] = make_float2(INFINITY, 0.f);
}

// Same contract as attn_bwd (csrc/attention.cu): delta = rowsum(dO * O), then the tcgen05 kernel, whose dQ partials
// (one per key tile) are summed by TMA reduce-adds into a zeroed fp32 buffer and stored as bf16 at the end.
void attn_bwd_tc(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k0, const at::Tensor& v0,
                 const c10::optional<at::Tensor>& k1, const c10::optional<at::Tensor>& v1, const at::Tensor& n0,
                 const at::Tensor& n1, const at::Tensor& o, const at::Tensor& lse, const at::Tensor& dq,
                 const at::Tensor& dk0, const at::Tensor& dv0, const c10::optional<at::Tensor>& dk1,
                 const c10::optional<at::Tensor>& dv1, int64_t Lq, int64_t L0, int64_t L1, double scale,
                 int64_t version) {
  TORCH_CHECK(q.is_cuda() && q.size(1) % 64 == 0, "attn_bwd_tc: head dim 64");
  TORCH_CHECK(n0.scalar_type() == at::kInt && n1.scalar_type() == at::kInt, "int32 key counts expected");
  for (const at::Tensor* t : {&dout, &o, &dq, &dk0, &dv0})
    TORCH_CHECK(t->dim() == 2 && t->stride(1) == 1 && t->stride(0) % 8 == 0 && t->scalar_type() == at::kBFloat16,
                "attn_bwd_tc: bf16 row-major views with 16-byte row strides expected");
  const at::cuda::CUDAGuard guard(q.device());
  const bool has1 = k1.has_value() && k1->defined() && L1 > 0;
  const int64_t B = q.size(0) / Lq, C = q.size(1);
  AttnTcBwdParams p{};
  p.n0 = n0.data_ptr<int>();
  p.n1 = n1.data_ptr<int>();
  p.Lq = (int)Lq;
  p.L0 = (int)L0;
  p.L1 = has1 ? (int)L1 : 0;
  p.H = (int)(C / 64);
  p.nt0 = (int)((L0 + atb::BK - 1) / atb::BK);
  p.nt1 = has1 ? (int)((L1 + atb::BK - 1) / atb::BK) : 0;
  p.nq = (int)((Lq + atb::BQ - 1) / atb::BQ);
  p.scale = (float)scale;
  p.scale_log2 = (float)scale * atc::kLog2e;
  p.lse = lse.data_ptr<float>();
  p.dk0 = reinterpret_cast<bf16*>(dk0.data_ptr());
  p.dv0 = reinterpret_cast<bf16*>(dv0.data_ptr());
  p.lddk0 = dk0.stride(0);
  p.lddv0 = dv0.stride(0);
  if (has1) {
    TORCH_CHECK(dk1.has_value() && dv1.has_value(), "attn_bwd_tc: dk1/dv1 required with a second key source");
    p.dk1 = reinterpret_cast<bf16*>(dk1->data_ptr());
    p.dv1 = reinterpret_cast<bf16*>(dv1->data_ptr());
    p.lddk1 = dk1->stride(0);
    p.lddv1 = dv1->stride(0);
  }
  p.err = status_word();
  auto s = at::cuda::getCurrentCUDAStream();
  at::Tensor delta, ldt;
  if (version == 1) {
    delta = at::empty({B, (int64_t)p.H, Lq}, q.options().dtype(at::kFloat));
    attn_delta(reinterpret_cast<const bf16*>(dout.data_ptr()), dout.stride(0),
               reinterpret_cast<const bf16*>(o.data_ptr()), o.stride(0), delta.data_ptr<float>(), (int)q.size(0),
               (int)Lq, p.H, s);
    p.delta = delta.data_ptr<float>();
  } else {
    const int64_t Lqp = (int64_t)p.nq * atb::BQ;
    ldt = at::empty({B, (int64_t)p.H, Lqp, 2}, q.options().dtype(at::kFloat));
    const int64_t n = B * Lq * p.H * 8 + B * p.H * (Lqp - Lq);
    attn_ld8_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<const bf16*>(dout.data_ptr()), dout.stride(0), reinterpret_cast<const bf16*>(o.data_ptr()),
        o.stride(0), lse.data_ptr<float>(), reinterpret_cast<float2*>(ldt.data_ptr()), (int)B, p.H, (int)Lq, (int)Lqp);
    NG_LAUNCH_CHECK();
  }
  CUtensorMap mq = make_tmap_bf16(q.data_ptr(), C, Lq, B, q.stride(0), q.stride(0) * Lq, 64, 128);
  CUtensorMap mdo = make_tmap_bf16(dout.data_ptr(), C, Lq, B, dout.stride(0), dout.stride(0) * Lq, 64, 128);
  CUtensorMap mk0 = seq_map(k0, L0), mv0 = seq_map(v0, L0);
  CUtensorMap mk1 = has1 ? seq_map(*k1, L1) : mk0, mv1 = has1 ? seq_map(*v1, L1) : mv0;
  if (version >= 3 && p.nq <= ab3::MAXQ) {
    // dQ accumulates in tensor memory: no fp32 buffer, no reduce-adds, no store pass
    AttnTcBwd3Params p3{};
    p3.n0 = p.n0;
    p3.n1 = p.n1;
    p3.Lq = p.Lq;
    p3.L0 = p.L0;
    p3.L1 = p.L1;
    p3.H = p.H;
    p3.nt0 = p.nt0;
    p3.nt1 = p.nt1;
    p3.nq = p.nq;
    p3.items = (int)B * p.H;
    p3.scale = p.scale;
    p3.scale_log2 = p.scale_log2;
    p3.ld = reinterpret_cast<const float2*>(ldt.data_ptr());
    p3.dq = reinterpret_cast<bf16*>(dq.data_ptr());
    p3.lddq = dq.stride(0);
    p3.dk0 = p.dk0;
    p3.dv0 = p.dv0;
    p3.dk1 = p.dk1;
    p3.dv1 = p.dv1;
    p3.lddk0 = p.lddk0;
    p3.lddv0 = p.lddv0;
    p3.lddk1 = p.lddk1;
    p3.lddv1 = p.lddv1;
    p3.err = p.err;
    static bool attr3 = false;
    static int sms3 = 0;
    if (!attr3) {
      cudaFuncSetAttribute(attn_bwd_tc3_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ab3::SMEM);
      cudaFuncSetAttribute(attn_bwd_tc3_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ab3::SMEM);
      cudaDeviceGetAttribute(&sms3, cudaDevAttrMultiProcessorCount, q.get_device());
      attr3 = true;
    }
    const int grid = std::max(1, std::min(p3.items, sms3));
    p3.prof = g_attn_prof;
    if (g_attn_prof != nullptr)
      attn_bwd_tc3_kernel<true><<<grid, ab3::THREADS, ab3::SMEM, s>>>(mq, mdo, mk0, mv0, mk1, mv1, p3);
    else
      attn_bwd_tc3_kernel<false><<<grid, ab3::THREADS, ab3::SMEM, s>>>(mq, mdo, mk0, mv0, mk1, mv1, p3);
    NG_LAUNCH_CHECK();
    return;
  }
  at::Tensor acc = at::empty({q.size(0), C}, q.options().dtype(at::kFloat));
  cudaMemsetAsync(acc.data_ptr(), 0, acc.numel() * sizeof(float), s);
  CUtensorMap mdq = make_tmap_f32_box(acc.data_ptr(), C, Lq, B, C, C * Lq, 32, 32);
  if (version == 1) {
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, atb::SMEM);
      attr = true;
    }
    dim3 grid((unsigned)(p.nt0 + p.nt1), (unsigned)(B * p.H));
    attn_bwd_tc_kernel<<<grid, atb::THREADS, atb::SMEM, s>>>(mq, mdo, mk0, mv0, mk1, mv1, mdq, p);
    NG_LAUNCH_CHECK();
  } else {
    AttnTcBwd2Params p2{};
    p2.n0 = p.n0;
    p2.n1 = p.n1;
    p2.Lq = p.Lq;
    p2.L0 = p.L0;
    p2.L1 = p.L1;
    p2.H = p.H;
    p2.nt0 = p.nt0;
    p2.nt1 = p.nt1;
    p2.nq = p.nq;
    p2.items = (int)B * p.H * (p.nt0 + p.nt1);
    p2.scale = p.scale;
    p2.scale_log2 = p.scale_log2;
    p2.ld = reinterpret_cast<const float2*>(ldt.data_ptr());
    p2.dk0 = p.dk0;
    p2.dv0 = p.dv0;
    p2.dk1 = p.dk1;
    p2.dv1 = p.dv1;
    p2.lddk0 = p.lddk0;
    p2.lddv0 = p.lddv0;
    p2.lddk1 = p.lddk1;
    p2.lddv1 = p.lddv1;
    p2.err = p.err;
    static bool attr2 = false;
    static int sms = 0;
    if (!attr2) {
      cudaFuncSetAttribute(attn_bwd_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ab2::SMEM);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, q.get_device());
      attr2 = true;
    }
    const int grid = std::max(1, std::min(p2.items, sms));
    attn_bwd_tc2_kernel<<<grid, ab2::THREADS, ab2::SMEM, s>>>(mq, mdo, mk0, mv0, mk1, mv1, mdq, p2);
    NG_LAUNCH_CHECK();
  }
  const int64_t n8 = q.size(0) * (C / 8);
  dq_store_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(acc.data_ptr<float>(),
                                                               reinterpret_cast<bf16*>(dq.data_ptr()), dq.stride(0),
                                                               q.size(0), (int)C);
  NG_LAUNCH_CHECK();
}

}  // namespace ng
