// Persistent tcgen05 GEMM for sm_100a: D[M, N] = A[M, K] * B[N, K]^T in bf16 with an fp32 accumulator in TMEM.
//
// Replaces every nn.Linear of the reference's JiT-T2I (cuBLAS under autocast, reference
// baselines/PixelGen/src/models/transformer/JiT_T2I.py:114-311) in its three forms:
//   forward  Y  = X  W^T     A K-major ([M, K] row-major), B K-major ([N, K] row-major)
//   dgrad    dX = dY W       A K-major, B MN-major ([K, N] row-major)
//   wgrad    dW = dY^T X     A MN-major ([K, M] row-major), B MN-major
// and the Newton-Schulz GEMM chain of Muon (reference baselines/PixelGen/src/optim/muon.py:64-86) through the
// batched alpha/beta epilogue.
//
// Structure (one CTA per SM, persistent over output tiles of 128 x 256):
//   warp 0      TMA producer: 4-stage ring of (A 128x64, B 256x64) bf16 tiles, 128-byte swizzle, one CTA per load
//   warp 1      TMEM owner and MMA issuer: tcgen05.mma M=128 N=256 K=16, one elected thread
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (double-buffered in TMEM, 2 x 256 columns), fused
//               elementwise work, vector stores to global memory
// The epilogue of tile i overlaps the MMAs of tile i+1.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>

#include "common.cuh"
#include "gemm.h"
#include "status.h"

namespace ng {

namespace gemm_cfg {
constexpr int BM = 128, BN = 256, BK = 64;
constexpr int A_BYTES = BM * BK * 2;  // 16 KiB
constexpr int B_BYTES = BN * BK * 2;  // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 320;  // producer, MMA, 8 epilogue warps (two per TMEM lane quarter)
constexpr int TMEM_COLS = 512;
// MXFP8 (block-scaled e4m3) tiles: 128 x 256 x 128 bytes per stage (the bf16 tile's bytes), plus the stage's scale
// factors: one 512-byte block for A's 128 rows and two for B's 256 rows. Both accumulators (256 columns each) and the
// 12 scale-factor columns must fit the 512 TMEM columns, so the second accumulator starts at column 224 and shares the
// first one's last 32 columns: the epilogue reads that shared chunk first and releases it (barrier `ovl`) before the
// rest of the tile, so the next tile's MMAs wait for one chunk read, not for the whole epilogue.
constexpr int MX_BK = 128;      // K elements (bytes) per stage
constexpr int MX_SF_STAGE = 1536;
constexpr int MX_ACC1 = 224;    // TMEM column of the second accumulator
constexpr int MX_SFA_COL = 480;  // 4 columns: A's scale factors of the stage (32 lanes x 4 row groups x 4 k-blocks)
constexpr int MX_SFB_COL = 488;  // 8 columns: B's scale factors (two 128-row blocks)
}  // namespace gemm_cfg

// Per-epilogue shared-memory plan. Epilogues that read inputs or write several outputs per tile (SwiGLU forward and
// backward, the gated residual) trade one mainloop stage (48 KiB) for a deeper epilogue pipeline: a ring of IN_RING
// prefetched input tiles and two output slots, so neither input latency nor store drain sits on the critical path.
// PAIR: the CTA-pair kernel (cta_group::2, 256 x 256 tiles per pair): a stage holds this CTA's 128 rows of A and 128
// columns of B (32 KiB), so the ring is deeper.
// MX: e4m3 operands with block scales (K-major A and B); the scale factors take 1.5 KiB per stage per CTA, so the
// ring has 3 stages (one CTA, 49.5 KiB a stage) or 4-5 (CTA pairs, 33.5 KiB a stage).
template <int EPI, bool PAIR = false, bool MX = false>
struct EpiCfg {
  static constexpr bool HEAVY = EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_BWD || EPI == EPI_GATED;
  static constexpr int STAGE_BYTES = PAIR ? gemm_cfg::A_BYTES + gemm_cfg::B_BYTES / 2 : gemm_cfg::STAGE_BYTES;
  // SwiGLU backward reads two input tiles per chunk: with pairs it keeps two chunks of inputs in flight (one stage
  // fewer in the mainloop ring)
  static constexpr int STAGES = MX ? (PAIR ? ((EPI == EPI_GATED || EPI == EPI_SWIGLU_BWD) ? 4 : 5) : 3)
                                   : PAIR ? (EPI == EPI_SWIGLU_BWD ? 4 : (HEAVY ? 5 : 6)) : (HEAVY ? 3 : 4);
  static constexpr int SF_BYTES = MX ? STAGES * gemm_cfg::MX_SF_STAGE : 0;
  // one output slot holds every 32x32 output tile of a chunk (bf16 2 KiB, fp32 4 KiB)
  static constexpr int OUT_SLOT = EPI == EPI_SWIGLU ? 6144
                                  : (EPI == EPI_F32 || EPI == EPI_GATED || EPI == EPI_SWIGLU_BWD) ? 4096
                                                                                                  : 2048;
  static constexpr int OUT_SLOTS = (EPI == EPI_BF16) ? 2 : 1;
  static constexpr int IN_SLOT = EPI == EPI_SWIGLU_BWD ? 4096 : (EPI == EPI_GATED || EPI == EPI_AXPBY) ? 2048 : 0;
  static constexpr int IN_RING =
      IN_SLOT == 0 ? 0 : ((EPI == EPI_GATED || (PAIR && !MX && EPI == EPI_SWIGLU_BWD)) ? 2 : 1);
  static constexpr int WARP_BYTES = (OUT_SLOTS * OUT_SLOT + IN_RING * IN_SLOT + 1023) / 1024 * 1024;
  static constexpr int EPI_BYTES = 8 * WARP_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + SF_BYTES + 1024 /*align slack*/ + 512 /*barriers*/;
  static_assert(SMEM <= 232448, "shared memory budget of one sm_100 CTA");
};

struct EpiParams {
  int M, N, K, batch;
  int half_n;  // SwiGLU: column offset of the second (x2) half in the pre-activation / the W12 rows
  void* out;
  int64_t ldo, out_bs;
  void* out2;
  int64_t ldo2;
  const float* bias;
  const __nv_bfloat16* res;
  int64_t ldr, res_bs;
  const __nv_bfloat16* gate;
  int64_t ldg;
  int rows_per_group;
  const int* seg;
  const __nv_bfloat16* aux;
  int64_t ld_aux;
  float alpha, beta;
  int accumulate;
  int k_splits;      // >1: split-K, each split writes its own fp32 slice out + split * out_bs
  int kb_per_split;  // k-blocks (of BK) per split
  const uint8_t* sfa;  // MX: scale-factor blocks of A: [ceil(M / 128) row blocks][K / 128][512 bytes]
  const uint8_t* sfb;  // MX: scale-factor blocks of B (row blocks of the B tensor's rows)
  uint8_t* act_q;      // MX SwiGLU (optional): act [M, half_n] in e4m3, and its scale blocks
  uint8_t* act_sf;
  int* err;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& b, int& mb, int& nb) {
  const int per_batch = num_m * num_n;
  b = t / per_batch;
  int r = t - b * per_batch;
  constexpr int GROUP_M = 8;
  const int per_group = GROUP_M * num_n;
  const int g = r / per_group;
  const int first_m = g * GROUP_M;
  const int gsize = min(num_m - first_m, GROUP_M);
  const int rr = r - g * per_group;
  mb = first_m + rr % gsize;
  nb = rr / gsize;
}

template <int EPI>
__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const float (&v)[32], int col0, int N) {
  if (col0 + 32 <= N) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 w;
      w.x = pack_bf16(v[8 * j + 0], v[8 * j + 1]);
      w.y = pack_bf16(v[8 * j + 2], v[8 * j + 3]);
      w.z = pack_bf16(v[8 * j + 4], v[8 * j + 5]);
      w.w = pack_bf16(v[8 * j + 6], v[8 * j + 7]);
      d4[j] = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) dst[j] = __float2bfloat16_rn(v[j]);
  }
}

__device__ __forceinline__ void load_row_bf16(const __nv_bfloat16* src, float (&v)[32], int col0, int N) {
  if (col0 + 32 <= N) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 w = s4[j];
      v[8 * j + 0] = bf16_bits_lo(w.x);
      v[8 * j + 1] = bf16_bits_hi(w.x);
      v[8 * j + 2] = bf16_bits_lo(w.y);
      v[8 * j + 3] = bf16_bits_hi(w.y);
      v[8 * j + 4] = bf16_bits_lo(w.z);
      v[8 * j + 5] = bf16_bits_hi(w.z);
      v[8 * j + 6] = bf16_bits_lo(w.w);
      v[8 * j + 7] = bf16_bits_hi(w.w);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (col0 + j < N) ? __bfloat162float(src[j]) : 0.0f;
  }
}

__device__ __forceinline__ void load_bias(const float* bias, float (&bv)[32], int col0, int N) {
  if (bias == nullptr) {
#pragma unroll
    for (int j = 0; j < 32; ++j) bv[j] = 0.f;
    return;
  }
  if (col0 + 32 <= N) {
    const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 w = __ldg(b4 + j);
      bv[4 * j] = w.x;
      bv[4 * j + 1] = w.y;
      bv[4 * j + 2] = w.z;
      bv[4 * j + 3] = w.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) bv[j] = (col0 + j < N) ? bias[col0 + j] : 0.f;
  }
}

// Epilogue tiles are 32 rows x 32 columns. bf16: 64-byte rows with the 64-byte TMA swizzle (16-byte chunk j of row r
// at chunk j ^ ((r >> 1) & 3)); fp32: 128-byte rows with the 128-byte swizzle (chunk j at j ^ (r & 7)). A thread owns
// one row, so a warp's 16-byte accesses hit 8 distinct bank groups per quarter-warp (conflict-free).
__device__ __forceinline__ uint32_t sw64(int r, int j) { return r * 64 + ((j ^ ((r >> 1) & 3)) << 4); }
__device__ __forceinline__ uint32_t sw128(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

__device__ __forceinline__ void st_tile_bf16(uint8_t* buf, int r, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 w;
    w.x = pack_bf16(v[8 * j + 0], v[8 * j + 1]);
    w.y = pack_bf16(v[8 * j + 2], v[8 * j + 3]);
    w.z = pack_bf16(v[8 * j + 4], v[8 * j + 5]);
    w.w = pack_bf16(v[8 * j + 6], v[8 * j + 7]);
    *reinterpret_cast<uint4*>(buf + sw64(r, j)) = w;
  }
}
__device__ __forceinline__ void ld_tile_bf16(const uint8_t* buf, int r, float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 w = *reinterpret_cast<const uint4*>(buf + sw64(r, j));
    v[8 * j + 0] = bf16_bits_lo(w.x);
    v[8 * j + 1] = bf16_bits_hi(w.x);
    v[8 * j + 2] = bf16_bits_lo(w.y);
    v[8 * j + 3] = bf16_bits_hi(w.y);
    v[8 * j + 4] = bf16_bits_lo(w.z);
    v[8 * j + 5] = bf16_bits_hi(w.z);
    v[8 * j + 6] = bf16_bits_lo(w.w);
    v[8 * j + 7] = bf16_bits_hi(w.w);
  }
}
__device__ __forceinline__ void st_tile_f32(uint8_t* buf, int r, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4*>(buf + sw128(r, j)) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// PAIR = true: launched as 2-CTA clusters; CTA r of a pair computes rows [256 mb + 128 r, +128) of a 256 x 256 tile.
// Its TMA warp loads its 128 rows of A and its 128 columns of B (counted on CTA 0's `full` barrier), CTA 0's MMA
// thread issues M = 256 tcgen05.mma.cta_group::2 over both CTAs' shared memory into both CTAs' TMEM and releases the
// stages / signals the accumulators in both CTAs; each CTA's epilogue drains its own rows and frees the accumulator
// on CTA 0's barrier. Per CTA and k-block 32 KiB are loaded instead of 48 KiB.
template <int AMN, int BMN, int EPI, bool PAIR, bool MX>
__global__ void __launch_bounds__(gemm_cfg::THREADS, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmOut2,
                        const __grid_constant__ CUtensorMap tmRes, const __grid_constant__ CUtensorMap tmAux,
                        const __grid_constant__ CUtensorMap tmSfa, const __grid_constant__ CUtensorMap tmSfb,
                        const EpiParams p) {
  using namespace gemm_cfg;
  static_assert(!MX || (AMN == 0 && BMN == 0), "MX tiles: K-major A and B");
  using Cfg = EpiCfg<EPI, PAIR, MX>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int SB = Cfg::STAGE_BYTES;
  constexpr int BMP = PAIR ? 2 * BM : BM;  // rows of one tile (of the pair)
  constexpr int BKE = MX ? MX_BK : BK;     // K elements per stage
  constexpr int ACC_STRIDE = MX ? MX_ACC1 : BN;  // TMEM column distance of the two accumulators
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sf_smem = smem + STAGES * SB + Cfg::EPI_BYTES;  // MX: [STAGES][1536] scale-factor blocks
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * SB + Cfg::EPI_BYTES + Cfg::SF_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* in_bar = drain + 1;  // [8 epilogue warps][2]: input ring slots
  uint64_t* ovl = in_bar + 16;    // MX: [2] the chunk an accumulator shares with the other one has been read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ovl + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = PAIR ? cluster_ctarank() : 0;
  const int tile0 = PAIR ? blockIdx.x >> 1 : blockIdx.x;  // this CTA's (pair's) first tile; stride = #clusters
  const int tstep = PAIR ? gridDim.x >> 1 : gridDim.x;
  // SwiGLU tiles cover 128 output columns of each half: the MMA's N extent is still 256
  const int num_m = (p.M + BMP - 1) / BMP;
  const int num_n = (EPI == EPI_SWIGLU) ? (p.half_n + 127) / 128 : (p.N + BN - 1) / BN;
  const int num_k = (p.K + BKE - 1) / BKE;
  const int splits = p.k_splits > 1 ? p.k_splits : 1;
  const int kps = splits > 1 ? p.kb_per_split : num_k;
  const int total = p.batch * splits * num_m * num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], PAIR ? 16 : 8);  // the epilogue warps of both CTAs free CTA 0's accumulators
    }
    mbar_init(drain, 1);
    for (int e = 0; e < 16; ++e) mbar_init(&in_bar[e], 1);
    mbar_init(&ovl[0], PAIR ? 16 : 8);  // (a pair: the epilogue warps of both CTAs)
    mbar_init(&ovl[1], PAIR ? 16 : 8);
    *abort_flag = 0;
    if (PAIR)
      fence_mbarrier_init_cluster();
    else
      fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
    if (MX && PAIR) {
      tma_prefetch_map(&tmSfa);
      tma_prefetch_map(&tmSfb);
    }
  }
  if (warp >= 2 && lane == 0) {
    tma_prefetch_map(&tmOut);
    if (EPI == EPI_GATED || EPI == EPI_SWIGLU) tma_prefetch_map(&tmOut2);
    if (EPI == EPI_GATED || EPI == EPI_AXPBY) tma_prefetch_map(&tmRes);
    if (EPI == EPI_SWIGLU_BWD) tma_prefetch_map(&tmAux);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the peer's barriers are initialised before anything signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;  // stages filled since the start (for draining on abort)
      for (int t = tile0; t < total && !*abort_flag; t += tstep) {
        int bs, mb, nb;
        tile_coords(t, num_m, num_n, bs, mb, nb);
        const int b = bs / splits, sp = bs - b * splits;
        const int kb0 = sp * kps, kb1 = min(num_k, kb0 + kps);
        const int arow = mb * BMP + (int)crank * BM;  // this CTA's first row of A
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.err, kErrWaitEmpty)) break;
          uint8_t* sA = smem + stage * SB;
          uint8_t* sB = sA + A_BYTES;
          const int k0 = kb * BKE;
          if (MX && PAIR) {
            // this CTA's 128 rows of A and its 128 rows (half) of B, its A scale block and BOTH B scale blocks (the
            // M = 256 MMA reads all 256 columns' scales from each CTA's tensor memory); the scale blocks come by tensor
            // TMA so that, like the operand tiles, their bytes count on CTA 0's barrier
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            const int rb = EPI == EPI_SWIGLU ? (crank == 0 ? nb * 128 : p.half_n + nb * 128) : nb * BN + (int)crank * 128;
            const int sb0 = EPI == EPI_SWIGLU ? nb : 2 * nb;
            const int sb1 = EPI == EPI_SWIGLU ? p.half_n / 128 + nb : 2 * nb + 1;
            uint8_t* sf = sf_smem + stage * MX_SF_STAGE;
            if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (SB + MX_SF_STAGE));
            tma_load_3d_pair(&tmA, fb, sA, k0, arow, 0);
            tma_load_3d_pair(&tmB, fb, sB, k0, rb, 0);
            tma_load_3d_pair(&tmSfa, fb, sf, 0, kb, arow / 128);
            tma_load_3d_pair(&tmSfb, fb, sf + 512, 0, kb, sb0);
            tma_load_3d_pair(&tmSfb, fb, sf + 1024, 0, kb, sb1);
          } else if (MX) {
            // A rows [arow, +128) and B rows of the tile, 128 e4m3 values of K each, plus their scale-factor blocks
            const int kt = num_k;  // scale-factor blocks per row block
            const int r0 = EPI == EPI_SWIGLU ? nb * 128 : nb * BN;
            const int r1 = EPI == EPI_SWIGLU ? p.half_n + nb * 128 : nb * BN + 128;
            uint8_t* sf = sf_smem + stage * MX_SF_STAGE;
            mbar_arrive_expect_tx(&full[stage], SB + MX_SF_STAGE);
            tma_load_3d(&tmA, &full[stage], sA, k0, arow, 0);
            tma_load_3d(&tmB, &full[stage], sB, k0, r0, 0);
            tma_load_3d(&tmB, &full[stage], sB + 16384, k0, r1, 0);
            bulk_load(sf, p.sfa + ((int64_t)mb * kt + kb) * 512, 512, &full[stage]);
            bulk_load(sf + 512, p.sfb + ((int64_t)(r0 / 128) * kt + kb) * 512, 512, &full[stage]);
            bulk_load(sf + 1024, p.sfb + ((int64_t)(r1 / 128) * kt + kb) * 512, 512, &full[stage]);
          } else if (PAIR) {
            // both CTAs' bytes are counted on CTA 0's full barrier; only CTA 0 announces them
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * SB);
            if (AMN == 0) {
              tma_load_3d_pair(&tmA, fb, sA, k0, arow, b);
            } else {
              tma_load_3d_pair(&tmA, fb, sA, arow, k0, b);
              tma_load_3d_pair(&tmA, fb, sA + 8192, arow + 64, k0, b);
            }
            if (BMN == 0) {
              const int r0 = EPI == EPI_SWIGLU ? (crank == 0 ? nb * 128 : p.half_n + nb * 128)
                                               : nb * BN + (int)crank * 128;
              tma_load_3d_pair(&tmB, fb, sB, k0, r0, b);
            } else {
              tma_load_3d_pair(&tmB, fb, sB, nb * BN + (int)crank * 128, k0, b);
              tma_load_3d_pair(&tmB, fb, sB + 8192, nb * BN + (int)crank * 128 + 64, k0, b);
            }
          } else {
            mbar_arrive_expect_tx(&full[stage], SB);
            if (AMN == 0) {
              tma_load_3d(&tmA, &full[stage], sA, k0, arow, b);
            } else {
              tma_load_3d(&tmA, &full[stage], sA, arow, k0, b);
              tma_load_3d(&tmA, &full[stage], sA + 8192, arow + 64, k0, b);
            }
            if (BMN == 0) {
              int r0, r1;
              if (EPI == EPI_SWIGLU) {
                r0 = nb * 128;
                r1 = p.half_n + nb * 128;
              } else {
                r0 = nb * BN;
                r1 = nb * BN + 128;
              }
              tma_load_3d(&tmB, &full[stage], sB, k0, r0, b);
              tma_load_3d(&tmB, &full[stage], sB + 16384, k0, r1, b);
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j) tma_load_3d(&tmB, &full[stage], sB + j * 8192, nb * BN + 64 * j, k0, b);
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag && (!PAIR || crank == 0)) {
        // unwinding: let the copies already issued land before the CTA's shared memory goes away (for a pair, CTA 0's
        // full barriers count both CTAs' copies)
        const uint64_t t0 = globaltimer_ns();
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < min(issued, STAGES); ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          while (!mbar_try_wait(&full[s], ph)) {
            if (globaltimer_ns() - t0 > NG_WAIT_BUDGET_NS) {
              raise_error(p.err, kErrWaitDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0 && crank == 0) {
      constexpr uint32_t idesc = MX ? idesc_mxf8_f32(BMP, BN) : idesc_bf16_f32(BMP, BN, AMN, BMN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool issued_any = false;
      // release / signal a barrier of this CTA and, for a pair, the same barrier of the peer
      auto commit_both = [&](uint64_t* bar) {
        if (PAIR) {
          umma_commit_pair(smem_u32(bar));
          umma_commit_pair(mapa_shared(smem_u32(bar), 1));
        } else {
          umma_commit(bar);
        }
      };
      for (int t = tile0; t < total && !*abort_flag; t += tstep, ++it) {
        const int a = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[a], aph ^ 1, abort_flag, p.err, kErrWaitAccEmpty)) break;
        // MX: the previous tile's accumulator shares 32 columns with this one; its epilogue has read them
        if (MX && it > 0 && !mbar_wait(&ovl[a ^ 1], ((it - 1) >> 1) & 1, abort_flag, p.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * ACC_STRIDE;
        bool ok = true;
        const int sp = (t / (num_m * num_n)) % splits;
        const int kb0 = sp * kps, kb1 = min(num_k, kb0 + kps);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * SB);
          const uint32_t sb = sa + A_BYTES;
          if (MX) {
            // this stage's scale factors into TMEM (executed in order with the MMAs before and after), then four
            // K = 32 MMAs, each using scale-factor byte k of every 32-bit TMEM word
            const uint32_t ssf = smem_u32(sf_smem + stage * MX_SF_STAGE);
            if (PAIR) {
              tmem_cp_32x128_x4_pair(tmem_base + MX_SFA_COL, smem_desc_sf(ssf));
              tmem_cp_32x128_x4_pair(tmem_base + MX_SFB_COL, smem_desc_sf(ssf + 512));
              tmem_cp_32x128_x4_pair(tmem_base + MX_SFB_COL + 4, smem_desc_sf(ssf + 1024));
            } else {
              tmem_cp_32x128_x4(tmem_base + MX_SFA_COL, smem_desc_sf(ssf));
              tmem_cp_32x128_x4(tmem_base + MX_SFB_COL, smem_desc_sf(ssf + 512));
              tmem_cp_32x128_x4(tmem_base + MX_SFB_COL + 4, smem_desc_sf(ssf + 1024));
            }
#pragma unroll
            for (int k = 0; k < MX_BK / 32; ++k) {
              const uint64_t da = smem_desc_sw128(sa + k * 32, 16, 1024);
              const uint64_t db = smem_desc_sw128(sb + k * 32, 16, 1024);
              const uint32_t id = idesc | ((uint32_t)k << 29) | ((uint32_t)k << 4);
              const uint32_t sfa = (tmem_base + MX_SFA_COL) | ((uint32_t)k << 30);
              const uint32_t sfb = (tmem_base + MX_SFB_COL) | ((uint32_t)k << 30);
              if (PAIR)
                umma_mxf8_pair(d_tmem, da, db, id, sfa, sfb, (kb != kb0 || k != 0) ? 1u : 0u);
              else
                umma_mxf8(d_tmem, da, db, id, sfa, sfb, (kb != kb0 || k != 0) ? 1u : 0u);
            }
          }
#pragma unroll
          for (int k = 0; k < (MX ? 0 : BK / 16); ++k) {
            const uint64_t da = AMN == 0 ? smem_desc_sw128(sa + k * 32, 16, 1024)
                                         : smem_desc_sw128(sa + k * 2048, 8192, 1024);
            const uint64_t db = BMN == 0 ? smem_desc_sw128(sb + k * 32, 16, 1024)
                                         : smem_desc_sw128(sb + k * 2048, 8192, 1024);
            if (PAIR)
              umma_f16_pair(d_tmem, da, db, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
            else
              umma_f16(d_tmem, da, db, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          issued_any = true;
          commit_both(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        commit_both(&acc_full[a]);
      }
      if (*abort_flag && issued_any) {
        // unwinding: wait for the MMAs in flight before TMEM is released
        if (PAIR)
          umma_commit_pair(smem_u32(drain));
        else
          umma_commit(drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (globaltimer_ns() - t0 > NG_WAIT_BUDGET_NS) {
            raise_error(p.err, kErrWaitDrain);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------------------------------------ epilogue
    // Warp e = warp - 2 may read TMEM lanes [32q, 32q+32), q = warp % 4: rows row0 .. row0+31 of each tile. A 32-column
    // chunk goes TMEM -> registers -> a swizzled smem tile -> one TMA store per output; inputs (the residual, C, or
    // the saved SwiGLU pre-activation) arrive by TMA loads into a ring of IN_RING slots that runs ahead of the chunk
    // being processed (across tiles), and outputs alternate between two slots, so neither the input latency nor the
    // drain of the previous stores is waited for. TMA clips rows/columns outside the tensors.
    // Two warps share each TMEM lane quarter and take alternate 32-column chunks of a tile (h = 0: even chunks).
    constexpr int NCH = (EPI == EPI_SWIGLU) ? 4 : BN / 32;
    constexpr int NCW = NCH / 2;  // chunks per warp per tile
    constexpr int R = Cfg::IN_RING;
    const int q = warp & 3, e = warp - 2, h = e >> 2;
    uint8_t* wbase = smem + STAGES * SB + e * Cfg::WARP_BYTES;
    uint8_t* ibase = wbase + Cfg::OUT_SLOTS * Cfg::OUT_SLOT;
    uint64_t* ibar = &in_bar[e * 2];
    const bool has_in = R > 0 && (EPI != EPI_AXPBY || p.beta != 0.f);
    const int my_tiles = tile0 < total ? (total - 1 - tile0) / tstep + 1 : 0;
    const int n_chunks = my_tiles * NCW;  // this warp's chunk sequence, in processing order
    // chunk of the k-th step of this warp's i-th tile: ascending, except that an MX tile in the first accumulator goes
    // backwards, so that its last chunk (the columns the second accumulator shares) is read first
    auto chunk_at = [&](int i, int k) { return (MX && !(i & 1)) ? h + 2 * (NCW - 1 - k) : h + 2 * k; };
    // issue the input loads of chunk L (linear index over this warp's chunks) into ring slot L % R
    auto issue_in = [&](int L) {
      if (!has_in || L >= n_chunks) return;
      const int i = L / NCW, c = chunk_at(i, L - (L / NCW) * NCW);
      int bs, mb, nb;
      tile_coords(tile0 + i * tstep, num_m, num_n, bs, mb, nb);
      const int row0 = mb * BMP + (int)crank * BM + q * 32;
      const int col = (EPI == EPI_SWIGLU ? nb * 128 : nb * BN) + c * 32;
      uint64_t* bar = &ibar[L % R];
      uint8_t* dst = ibase + (L % R) * Cfg::IN_SLOT;
      if (EPI == EPI_SWIGLU_BWD) {
        mbar_arrive_expect_tx(bar, 4096);
        tma_load_3d(&tmAux, bar, dst, col, row0, 0);
        tma_load_3d(&tmAux, bar, dst + 2048, p.half_n + col, row0, 0);
      } else {
        mbar_arrive_expect_tx(bar, 2048);
        tma_load_3d(&tmRes, bar, dst, col, row0, bs);
      }
    };
    if (lane == 0)
      for (int L = 0; L < R; ++L) issue_in(L);
    int it = 0, L = 0, oslot = 0;
    bool ok = true;
    for (int t = tile0; t < total && ok; t += tstep, ++it) {
      const int a = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      const bool got = __all_sync(0xffffffffu, mbar_wait(&acc_full[a], aph, abort_flag, p.err, kErrWaitAccFull));
      if (!got) break;
      tc_fence_after();
      int bs, mb, nb;
      tile_coords(t, num_m, num_n, bs, mb, nb);
      const int row0 = mb * BMP + (int)crank * BM + q * 32;
      const int row = row0 + lane;
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + a * ACC_STRIDE;
#pragma unroll 1
      for (int k = 0; k < NCW; ++k, ++L) {
        const int c = chunk_at(it, k);
        const int col = (EPI == EPI_SWIGLU ? nb * 128 : nb * BN) + c * 32;
        const bool live = col < ((EPI == EPI_SWIGLU) ? p.half_n : p.N);  // warp-uniform
        uint32_t r1[32], r2[32];
        __syncwarp();
        tmem_ld32(tb + c * 32, r1);
        if (EPI == EPI_SWIGLU) tmem_ld32(tb + 128 + c * 32, r2);
        tmem_wait_ld();
        if (MX && k == 0) {
          // the first chunk (which includes the shared columns) is in registers: the next tile may overwrite them
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (PAIR)
              mbar_arrive_cluster(mapa_shared(smem_u32(&ovl[a]), 0));
            else
              mbar_arrive(&ovl[a]);
          }
        }
        // per-sample gate / bias values (global, shared by the warp's lanes) before waiting for the inputs
        float gv[32], bv[32];
        if (live && (EPI == EPI_GATED || EPI == EPI_BF16)) load_bias(p.bias, bv, col, p.N);
        if (live && EPI == EPI_GATED) {
          const int crow = min(row, p.M - 1);
          const int grow = p.seg != nullptr ? p.seg[crow] : crow / p.rows_per_group;
          load_row_bf16(p.gate + (int64_t)grow * p.ldg + col, gv, col, p.N);
        }
        const uint8_t* ibuf = ibase + (L % (R > 0 ? R : 1)) * Cfg::IN_SLOT;
        if (has_in) {
          const bool arrived = mbar_wait(&ibar[L % R], (L / R) & 1, abort_flag, p.err, kErrWaitFull);
          __syncwarp();
          if (!arrived) {
            ok = false;
            break;
          }
        }
        // output slot: the stores last issued from it must have read it
        uint8_t* obuf = wbase + oslot * Cfg::OUT_SLOT;
        if (lane == 0) {
          if (Cfg::OUT_SLOTS == 2)
            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          else
            bulk_wait_read0();
        }
        __syncwarp();
        if (live) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r1[j]);
          if (EPI == EPI_BF16) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += bv[j];
            st_tile_bf16(obuf, lane, v);
          } else if (EPI == EPI_F32) {
            st_tile_f32(obuf, lane, v);
          } else if (EPI == EPI_AXPBY) {
            if (has_in) {
              float cv[32];
              ld_tile_bf16(ibuf, lane, cv);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = p.alpha * v[j] + p.beta * cv[j];
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = p.alpha * v[j];
            }
            st_tile_bf16(obuf, lane, v);
          } else if (EPI == EPI_GATED) {
            // y = acc + bias (kept for the backward); out = res + gate[sample] * y
            float rv[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = round_bf16(v[j] + bv[j]);
            st_tile_bf16(obuf + 2048, lane, v);
            ld_tile_bf16(ibuf, lane, rv);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = rv[j] + gv[j] * v[j];
            st_tile_bf16(obuf, lane, v);
          } else if (EPI == EPI_SWIGLU) {
            // accumulator columns [0,128) are x1 (gate half), [128,256) are x2 (up half)
            float x2[32], h[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              v[j] = round_bf16(v[j]);
              x2[j] = round_bf16(__uint_as_float(r2[j]));
              h[j] = round_bf16(v[j] * sigmoidf_(v[j])) * x2[j];
            }
            st_tile_bf16(obuf, lane, v);
            st_tile_bf16(obuf + 2048, lane, x2);
            st_tile_bf16(obuf + 4096, lane, h);
            if constexpr (MX) {
              // the MXFP8 copy of act for the next MX GEMM: this lane's 32 columns of its row are one scale block
              if (p.act_q != nullptr && row < p.M) {
                float am = 0.f;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  h[j] = round_bf16(h[j]);
                  am = fmaxf(am, fabsf(h[j]));
                }
                const int e = mx_scale_exp(am);
                const float inv = ldexpf(1.f, -e);
                uint4* dq = reinterpret_cast<uint4*>(p.act_q + (int64_t)row * p.half_n + col);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                  uint4 o;
                  o.x = e4m3x4(h[16 * j] * inv, h[16 * j + 1] * inv, h[16 * j + 2] * inv, h[16 * j + 3] * inv);
                  o.y = e4m3x4(h[16 * j + 4] * inv, h[16 * j + 5] * inv, h[16 * j + 6] * inv, h[16 * j + 7] * inv);
                  o.z = e4m3x4(h[16 * j + 8] * inv, h[16 * j + 9] * inv, h[16 * j + 10] * inv, h[16 * j + 11] * inv);
                  o.w = e4m3x4(h[16 * j + 12] * inv, h[16 * j + 13] * inv, h[16 * j + 14] * inv, h[16 * j + 15] * inv);
                  dq[j] = o;
                }
                p.act_sf[mx_sf_offset(row, col / 32, p.half_n / 128)] = (uint8_t)(e + 127);
              }
            }
          } else if (EPI == EPI_SWIGLU_BWD) {
            // v = d(act) for act columns [col, col+32); ibuf = the saved pre-activation tiles [x1 | x2]
            float x1[32], x2[32], d2[32];
            ld_tile_bf16(ibuf, lane, x1);
            ld_tile_bf16(ibuf + 2048, lane, x2);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float sg = sigmoidf_(x1[j]);
              d2[j] = v[j] * x1[j] * sg;
              v[j] = v[j] * x2[j] * (sg * (1.0f + x1[j] * (1.0f - sg)));
            }
            st_tile_bf16(obuf, lane, v);
            st_tile_bf16(obuf + 2048, lane, d2);
            if constexpr (MX) {
              // the MXFP8 copy of d(pre) = [d1 | d2] for the next MX dgrad (w12's): this lane's 32 columns of d1 and
              // of d2 are one scale block each, quantized from the bf16 values the tiles hold
              if (p.act_q != nullptr && row < p.M) {
                const int kb = 2 * p.half_n / 128;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                  float* h = half == 0 ? v : d2;
                  float am = 0.f;
#pragma unroll
                  for (int j = 0; j < 32; ++j) {
                    h[j] = round_bf16(h[j]);
                    am = fmaxf(am, fabsf(h[j]));
                  }
                  const int e = mx_scale_exp(am);
                  const float inv = ldexpf(1.f, -e);
                  const int c = half * p.half_n + col;
                  uint4* dq = reinterpret_cast<uint4*>(p.act_q + (int64_t)row * 2 * p.half_n + c);
#pragma unroll
                  for (int j = 0; j < 2; ++j) {
                    uint4 o;
                    o.x = e4m3x4(h[16 * j] * inv, h[16 * j + 1] * inv, h[16 * j + 2] * inv, h[16 * j + 3] * inv);
                    o.y = e4m3x4(h[16 * j + 4] * inv, h[16 * j + 5] * inv, h[16 * j + 6] * inv, h[16 * j + 7] * inv);
                    o.z = e4m3x4(h[16 * j + 8] * inv, h[16 * j + 9] * inv, h[16 * j + 10] * inv, h[16 * j + 11] * inv);
                    o.w = e4m3x4(h[16 * j + 12] * inv, h[16 * j + 13] * inv, h[16 * j + 14] * inv,
                                 h[16 * j + 15] * inv);
                    dq[j] = o;
                  }
                  p.act_sf[mx_sf_offset(row, c / 32, kb)] = (uint8_t)(e + 127);
                }
              }
            }
          }
          fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) {
          if (live) {
            if (EPI == EPI_BF16 || EPI == EPI_AXPBY) {
              tma_store_3d(&tmOut, obuf, col, row0, bs);
            } else if (EPI == EPI_F32) {
              if (p.accumulate)
                tma_reduce_add_3d(&tmOut, obuf, col, row0, bs);
              else
                tma_store_3d(&tmOut, obuf, col, row0, bs);
            } else if (EPI == EPI_GATED) {
              tma_store_3d(&tmOut2, obuf + 2048, col, row0, 0);
              tma_store_3d(&tmOut, obuf, col, row0, 0);
            } else if (EPI == EPI_SWIGLU) {
              tma_store_3d(&tmOut2, obuf, col, row0, 0);
              tma_store_3d(&tmOut2, obuf + 2048, p.half_n + col, row0, 0);
              tma_store_3d(&tmOut, obuf + 4096, col, row0, 0);
            } else if (EPI == EPI_SWIGLU_BWD) {
              tma_store_3d(&tmOut, obuf, col, row0, 0);
              tma_store_3d(&tmOut, obuf + 2048, p.half_n + col, row0, 0);
            }
          }
          bulk_commit();  // (an empty group keeps the two-slot accounting uniform)
          // this chunk's input slot has been read by every lane: refill it with the chunk R ahead
          if (R > 0) issue_in(L + R);
        }
        if (Cfg::OUT_SLOTS == 2) oslot ^= 1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[a]), 0));
        else
          mbar_arrive(&acc_empty[a]);
      }
    }
    // every store has finished before the CTA (and its shared memory) goes away; on an abort, the input loads still
    // in flight land first (bounded wait)
    if (lane == 0) {
      bulk_wait0();
      if (has_in && !ok) {
        const uint64_t t0 = globaltimer_ns();
        for (int k = L; k < min(L + R, n_chunks); ++k)
          while (!mbar_try_wait(&ibar[k % R], (k / R) & 1))
            if (globaltimer_ns() - t0 > NG_WAIT_BUDGET_NS) {
              raise_error(p.err, kErrWaitDrain);
              break;
            }
      }
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the peer no longer reads this CTA's shared memory or signals its barriers
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ============================================================================================================== host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && ptr != nullptr,
                "nano_gpic_b200: cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

static bool trace_on() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("NG_TRACE");
    v = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}
#define NG_TRACE(...)                   \
  do {                                  \
    if (trace_on()) {                   \
      fprintf(stderr, __VA_ARGS__);     \
      fflush(stderr);                   \
    }                                   \
  } while (0)

// cuTensorMapEncodeTiled is a driver-API call and needs a current context in the calling thread. A fresh autograd
// worker thread whose first CUDA work is this call has none (torch's device guard skips cudaSetDevice when the index
// already matches), and the driver then crashes; so make the primary context current once per thread.
static void ensure_context() {
  thread_local bool ready = false;
  if (ready) return;
  int dev = 0;
  TORCH_CHECK(cudaGetDevice(&dev) == cudaSuccess, "cudaGetDevice failed");
  TORCH_CHECK(cudaSetDevice(dev) == cudaSuccess, "cudaSetDevice failed");
  TORCH_CHECK(cudaFree(nullptr) == cudaSuccess, "CUDA context initialisation failed");
  ready = true;
}

// A 3-D tensor map (inner, outer, batch); inner is contiguous. ld / bstride in elements.
static CUtensorMap make_tmap(const void* ptr, CUtensorMapDataType dt, int esize, int64_t inner, int64_t outer,
                             int64_t batch, int64_t ld, int64_t bstride, int box_inner, int box_outer,
                             CUtensorMapSwizzle sw) {
  ensure_context();
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * esize), (cuuint64_t)((batch > 1 ? bstride : ld * outer) * esize)};
  cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  TORCH_CHECK(ptr != nullptr, "TMA operand is null");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK((ld * esize) % 16 == 0, "TMA row stride must be a multiple of 16 bytes, got ld=", ld);
  TORCH_CHECK(batch == 1 || (bstride * esize) % 16 == 0, "TMA batch stride must be a multiple of 16 bytes");
  NG_TRACE("[tmap] ptr=%p inner=%lld outer=%lld batch=%lld ld=%lld box=%dx%d\n", ptr, (long long)inner,
           (long long)outer, (long long)batch, (long long)ld, box_inner, box_outer);
  CUresult r = get_encode_fn()(&m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

// bf16 operand map with the 128-byte swizzle (the GEMM's A/B tiles).
CUtensorMap make_tmap_bf16(const void* ptr, int64_t inner, int64_t outer, int64_t batch, int64_t ld, int64_t bstride,
                           int box_inner, int box_outer) {
  return make_tmap(ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, inner, outer, batch, ld, bstride, box_inner, box_outer,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

// fp32 map with the 128-byte swizzle and a given box (inner box of 32 fp32 = 128 bytes).
CUtensorMap make_tmap_f32_box(const void* ptr, int64_t inner, int64_t outer, int64_t batch, int64_t ld,
                              int64_t bstride, int box_inner, int box_outer) {
  return make_tmap(ptr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, inner, outer, batch, ld, bstride, box_inner, box_outer,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

// 32 x 32 epilogue tile maps: bf16 with the 64-byte swizzle, fp32 with the 128-byte swizzle.
static CUtensorMap epi_map_bf16(const void* ptr, int64_t cols, int64_t rows, int64_t batch, int64_t ld, int64_t bs) {
  return make_tmap(ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows, batch, ld, bs, 32, 32,
                   CU_TENSOR_MAP_SWIZZLE_64B);
}
static CUtensorMap epi_map_f32(const void* ptr, int64_t cols, int64_t rows, int64_t batch, int64_t ld, int64_t bs) {
  return make_tmap(ptr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, cols, rows, batch, ld, bs, 32, 32,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

struct EpiMaps {
  CUtensorMap out, out2, res, aux, sfa, sfb;
};

// CTA pairs (cta_group::2) for GEMMs with at least two 128-row blocks; NG_GEMM_PAIR=0 or gemm_set_pair(0) turns them
// off (A/B timing, tests of both paths).
static int g_pair_mode = -1;
void gemm_set_pair(int64_t on) { g_pair_mode = on ? 1 : 0; }
bool gemm_use_pair(int64_t M) {
  if (g_pair_mode < 0) {
    const char* e = getenv("NG_GEMM_PAIR");
    g_pair_mode = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return g_pair_mode == 1 && M >= 256;
}

template <int AMN, int BMN, int EPI, bool PAIR, bool MX = false>
static void launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const EpiMaps& em, const EpiParams& p,
                     int64_t tiles, cudaStream_t s) {
  auto kern = gemm_tcgen05_kernel<AMN, BMN, EPI, PAIR, MX>;
  constexpr int smem = EpiCfg<EPI, PAIR, MX>::SMEM;
  static bool attr_set = false;
  static int max_clusters = 0;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(gemm_cfg::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  if (PAIR) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (PAIR) {
      cfg.gridDim = dim3(2 * (num_sms() / 2));
      cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg);
      if (max_clusters <= 0) max_clusters = num_sms() / 2;
    }
    attr_set = true;
  }
  // persistent: one CTA (pair) per SM (pair) that can be resident at once
  const int64_t units = PAIR ? std::min<int64_t>(tiles, max_clusters) : std::min<int64_t>(tiles, num_sms());
  cfg.gridDim = dim3((unsigned)(PAIR ? 2 * units : units));
  TORCH_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, em.out, em.out2, em.res, em.aux, em.sfa, em.sfb, p) == cudaSuccess,
              "gemm launch failed");
  NG_LAUNCH_CHECK();
}

template <int AMN, int BMN, bool PAIR>
static void dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const EpiMaps& em, const EpiParams& p,
                         int64_t tiles, cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return launch_t<AMN, BMN, EPI_BF16, PAIR>(ta, tb, em, p, tiles, s);
    case EPI_F32: return launch_t<AMN, BMN, EPI_F32, PAIR>(ta, tb, em, p, tiles, s);
    case EPI_AXPBY: return launch_t<AMN, BMN, EPI_AXPBY, PAIR>(ta, tb, em, p, tiles, s);
    case EPI_GATED: return launch_t<AMN, BMN, EPI_GATED, PAIR>(ta, tb, em, p, tiles, s);
    case EPI_SWIGLU: return launch_t<AMN, BMN, EPI_SWIGLU, PAIR>(ta, tb, em, p, tiles, s);
    case EPI_SWIGLU_BWD: return launch_t<AMN, BMN, EPI_SWIGLU_BWD, PAIR>(ta, tb, em, p, tiles, s);
    default: TORCH_CHECK(false, "unknown GEMM epilogue ", epi);
  }
}

template <bool PAIR>
static void dispatch_major(int a_mn, int b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                           const EpiMaps& em, const EpiParams& p, int64_t tiles, cudaStream_t s) {
  if (!a_mn && !b_mn)
    dispatch_epi<0, 0, PAIR>(epi, ta, tb, em, p, tiles, s);
  else if (!a_mn && b_mn)
    dispatch_epi<0, 1, PAIR>(epi, ta, tb, em, p, tiles, s);
  else if (a_mn && b_mn)
    dispatch_epi<1, 1, PAIR>(epi, ta, tb, em, p, tiles, s);
  else
    dispatch_epi<1, 0, PAIR>(epi, ta, tb, em, p, tiles, s);
}

void gemm_launch(const GemmArgs& g, cudaStream_t stream) {
  using namespace gemm_cfg;
  TORCH_CHECK(g.M > 0 && g.N > 0 && g.K > 0 && g.batch > 0, "empty GEMM");
  NG_TRACE("[gemm] M=%d N=%d K=%d batch=%d a_mn=%d b_mn=%d epi=%d lda=%lld ldb=%lld ldo=%lld splits=%d A=%p B=%p out=%p\n",
           g.M, g.N, g.K, g.batch, g.a_mn, g.b_mn, g.epi, (long long)g.lda, (long long)g.ldb, (long long)g.ldo,
           g.k_splits, g.A, g.B, g.out);
  const int64_t b_rows = g.b_rows > 0 ? g.b_rows : g.N;
  CUtensorMap ta, tb;
  if (g.mx) {
    // e4m3 operands, K-major, boxes of 128 bytes x 128 rows (the bf16 tile's bytes)
    TORCH_CHECK(!g.a_mn && !g.b_mn && g.batch == 1 && g.k_splits <= 1 && g.K % MX_BK == 0,
                "MXFP8 GEMM: K-major A and B, one batch, K a multiple of 128");
    TORCH_CHECK(g.epi == EPI_BF16 || g.epi == EPI_GATED || g.epi == EPI_SWIGLU || g.epi == EPI_SWIGLU_BWD,
                "MXFP8 GEMM: unsupported epilogue");
    TORCH_CHECK(g.epi != EPI_SWIGLU_BWD || (g.half_n == g.N && g.N % 128 == 0 && g.aux != nullptr),
                "MXFP8 SwiGLU backward: N = half width, a multiple of 128, and the saved pre-activation");
    TORCH_CHECK(g.sfa != nullptr && g.sfb != nullptr && (reinterpret_cast<uintptr_t>(g.sfa) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(g.sfb) & 15) == 0,
                "MXFP8 GEMM: 16-byte aligned scale factors expected");
    TORCH_CHECK(g.epi != EPI_SWIGLU || g.half_n % 128 == 0, "MXFP8 SwiGLU: half width a multiple of 128");
    ta = make_tmap(g.A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.K, g.M, 1, g.lda, 0, MX_BK, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    tb = make_tmap(g.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.K, b_rows, 1, g.ldb, 0, MX_BK, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    // operand tensor maps: K-major [rows, K] boxes of 64 x 128; MN-major [K, rows] boxes of 64 x 64
    ta = g.a_mn ? make_tmap_bf16(g.A, g.M, g.K, g.batch, g.lda, g.a_bs, 64, 64)
                : make_tmap_bf16(g.A, g.K, g.M, g.batch, g.lda, g.a_bs, 64, 128);
    tb = g.b_mn ? make_tmap_bf16(g.B, b_rows, g.K, g.batch, g.ldb, g.b_bs, 64, 64)
                : make_tmap_bf16(g.B, g.K, b_rows, g.batch, g.ldb, g.b_bs, 64, 128);
  }
  EpiParams p;
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.batch = g.batch;
  p.half_n = g.half_n;
  p.out = g.out;
  p.ldo = g.ldo;
  p.out_bs = g.out_bs;
  p.out2 = g.out2;
  p.ldo2 = g.ldo2;
  p.bias = g.bias;
  p.res = g.res;
  p.ldr = g.ldr;
  p.res_bs = g.res_bs;
  p.gate = g.gate;
  p.ldg = g.ldg;
  p.rows_per_group = g.rows_per_group > 0 ? g.rows_per_group : 1;
  p.seg = g.seg;
  p.aux = g.aux;
  p.ld_aux = g.ld_aux;
  p.alpha = g.alpha;
  p.beta = (g.res != nullptr) ? g.beta : 0.f;
  p.accumulate = g.accumulate;
  p.k_splits = g.k_splits > 1 ? g.k_splits : 1;
  p.kb_per_split = g.kb_per_split;
  p.sfa = static_cast<const uint8_t*>(g.sfa);
  p.sfb = static_cast<const uint8_t*>(g.sfb);
  p.act_q = static_cast<uint8_t*>(g.act_q);
  p.act_sf = static_cast<uint8_t*>(g.act_sf);
  p.err = g.err;
  // MX on CTA pairs: opt-in (NG_MX_PAIR=1) until validated on the GPU
  static const bool mx_pair = getenv("NG_MX_PAIR") != nullptr && getenv("NG_MX_PAIR")[0] == '1';
  const bool pair = gemm_use_pair(g.M) && (!g.mx || mx_pair);
  const int num_m = (g.M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM);
  const int num_n = g.epi == EPI_SWIGLU ? (g.half_n + 127) / 128 : (g.N + BN - 1) / BN;
  const int64_t tiles = (int64_t)g.batch * (g.k_splits > 1 ? g.k_splits : 1) * num_m * num_n;
  // epilogue maps: the output(s) and the input tiles the epilogue reads
  const int zb = g.k_splits > 1 ? g.k_splits : g.batch;
  EpiMaps em;
  if (g.epi == EPI_F32) {
    em.out = epi_map_f32(g.out, g.N, g.M, zb, g.ldo, g.out_bs);
  } else {
    const int64_t ocols = g.epi == EPI_SWIGLU ? g.half_n : (g.epi == EPI_SWIGLU_BWD ? 2 * (int64_t)g.half_n : g.N);
    em.out = epi_map_bf16(g.out, ocols, g.M, zb, g.ldo, g.out_bs);
  }
  em.out2 = em.res = em.aux = em.sfa = em.sfb = em.out;
  if (g.mx && pair) {
    // scale blocks as [row blocks][K / 128][128 x u32]: one 512-byte box per (k-block, row block)
    const int64_t kt = g.K / MX_BK;
    em.sfa = make_tmap(g.sfa, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, 128, kt, (g.M + 255) / 256 * 2, 128, kt * 128, 128, 1,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
    em.sfb = make_tmap(g.sfb, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, 128, kt, (b_rows + 255) / 256 * 2, 128, kt * 128, 128,
                       1, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (g.epi == EPI_GATED) em.out2 = epi_map_bf16(g.out2, g.N, g.M, 1, g.ldo2, 0);
  if (g.epi == EPI_SWIGLU) em.out2 = epi_map_bf16(g.out2, 2 * (int64_t)g.half_n, g.M, 1, g.ldo2, 0);
  if (g.epi == EPI_GATED || (g.epi == EPI_AXPBY && g.beta != 0.f && g.res != nullptr))
    em.res = epi_map_bf16(g.res, g.N, g.M, g.batch, g.ldr, g.res_bs);
  if (g.epi == EPI_SWIGLU_BWD) em.aux = epi_map_bf16(g.aux, 2 * (int64_t)g.half_n, g.M, 1, g.ld_aux, 0);
  NG_TRACE("[gemm]   maps ok, pair=%d tiles=%lld\n", (int)pair, (long long)tiles);
  if (g.mx && pair) {
    switch (g.epi) {
      case EPI_BF16: launch_t<0, 0, EPI_BF16, true, true>(ta, tb, em, p, tiles, stream); break;
      case EPI_GATED: launch_t<0, 0, EPI_GATED, true, true>(ta, tb, em, p, tiles, stream); break;
      case EPI_SWIGLU_BWD: launch_t<0, 0, EPI_SWIGLU_BWD, true, true>(ta, tb, em, p, tiles, stream); break;
      default: launch_t<0, 0, EPI_SWIGLU, true, true>(ta, tb, em, p, tiles, stream); break;
    }
  } else if (g.mx) {
    switch (g.epi) {
      case EPI_BF16: launch_t<0, 0, EPI_BF16, false, true>(ta, tb, em, p, tiles, stream); break;
      case EPI_GATED: launch_t<0, 0, EPI_GATED, false, true>(ta, tb, em, p, tiles, stream); break;
      case EPI_SWIGLU_BWD: launch_t<0, 0, EPI_SWIGLU_BWD, false, true>(ta, tb, em, p, tiles, stream); break;
      default: launch_t<0, 0, EPI_SWIGLU, false, true>(ta, tb, em, p, tiles, stream); break;
    }
  } else if (pair)
    dispatch_major<true>(g.a_mn, g.b_mn, g.epi, ta, tb, em, p, tiles, stream);
  else
    dispatch_major<false>(g.a_mn, g.b_mn, g.epi, ta, tb, em, p, tiles, stream);
  NG_TRACE("[gemm]   launched\n");
}

}  // namespace ng

// ======================================================================================================= torch glue
#include "status.h"

namespace ng {

// out[i] (+)= sum_s ws[s * n + i], splits summed in order (deterministic)
__global__ void splitk_reduce_kernel(const float4* __restrict__ ws, int splits, int64_t n4, float4* __restrict__ out,
                                     int accumulate) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  float4 a = accumulate ? out[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < splits; ++s) {
    const float4 v = ws[s * n4 + i];
    a.x += v.x;
    a.y += v.y;
    a.z += v.z;
    a.w += v.w;
  }
  out[i] = a;
}

static void splitk_reduce(const float* ws, int splits, int64_t n, float* out, bool accumulate, cudaStream_t s) {
  TORCH_CHECK(n % 4 == 0, "split-K reduce needs a multiple of 4 elements");
  const int64_t n4 = n / 4;
  splitk_reduce_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, s>>>(reinterpret_cast<const float4*>(ws), splits, n4,
                                                                   reinterpret_cast<float4*>(out), accumulate ? 1 : 0);
  NG_LAUNCH_CHECK();
}

static const void* ptr_or_null(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr;
}

// All strides are in elements; every tensor is addressed from its data_ptr (storage offset included).
void gemm_torch(const at::Tensor& A, bool a_mn, int64_t lda, int64_t a_bs, const at::Tensor& B, bool b_mn, int64_t ldb,
                int64_t b_bs, int64_t b_rows, const at::Tensor& out, int64_t ldo, int64_t out_bs, int64_t epi, int64_t M,
                int64_t N, int64_t K, int64_t batch, const c10::optional<at::Tensor>& out2, int64_t ldo2,
                const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& res, int64_t ldr,
                int64_t res_bs, const c10::optional<at::Tensor>& gate, int64_t ldg, int64_t rows_per_group,
                const c10::optional<at::Tensor>& aux, int64_t ld_aux, int64_t half_n, double alpha, double beta,
                bool accumulate, const c10::optional<at::Tensor>& seg) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && out.is_cuda(), "gemm: CUDA tensors expected");
  if (seg.has_value() && seg->defined())
    TORCH_CHECK(seg->is_cuda() && seg->scalar_type() == at::kInt && seg->is_contiguous() && seg->numel() == M &&
                    epi == EPI_GATED,
                "gemm: seg must be an [M] int32 CUDA tensor, for the gated epilogue");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands expected");
  if (bias.has_value() && bias->defined()) TORCH_CHECK(bias->scalar_type() == at::kFloat, "gemm: fp32 bias expected");
  const at::cuda::CUDAGuard guard(A.device());
  NG_TRACE("[gemm_torch] enter epi=%lld M=%lld N=%lld K=%lld\n", (long long)epi, (long long)M, (long long)N, (long long)K);
  if (trace_on()) {
    const cudaError_t pre = cudaDeviceSynchronize();
    NG_TRACE("[gemm_torch]   device state before: %s\n", cudaGetErrorString(pre));
  }
  GemmArgs g;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.batch = (int)batch;
  g.A = A.data_ptr();
  g.lda = lda;
  g.a_bs = a_bs;
  g.a_mn = a_mn;
  g.B = B.data_ptr();
  g.ldb = ldb;
  g.b_bs = b_bs;
  g.b_mn = b_mn;
  g.b_rows = b_rows;
  g.epi = (int)epi;
  g.out = out.data_ptr();
  g.ldo = ldo;
  g.out_bs = out_bs;
  g.out2 = const_cast<void*>(ptr_or_null(out2));
  g.ldo2 = ldo2;
  g.bias = static_cast<const float*>(ptr_or_null(bias));
  g.res = static_cast<const __nv_bfloat16*>(ptr_or_null(res));
  g.ldr = ldr;
  g.res_bs = res_bs;
  g.gate = static_cast<const __nv_bfloat16*>(ptr_or_null(gate));
  g.ldg = ldg;
  g.rows_per_group = (int)rows_per_group;
  g.seg = static_cast<const int*>(ptr_or_null(seg));
  g.aux = static_cast<const __nv_bfloat16*>(ptr_or_null(aux));
  g.ld_aux = ld_aux;
  g.half_n = (int)half_n;
  g.alpha = (float)alpha;
  g.beta = (float)beta;
  g.accumulate = accumulate ? 1 : 0;
  g.err = status_word();
  auto stream = at::cuda::getCurrentCUDAStream();
  // Weight gradients have few output tiles (a 3072 x 1024 dW is 48 CTA-pair tiles for 74 pair slots: one wave at
  // 65 %) but a long reduction (all tokens): split K, each split writes an fp32 slice, then one ordered reduction adds
  // the slices (deterministic). The split count minimises a wave model: waves(tiles x s) x k-blocks per split, plus
  // the reduction's traffic ((s + 2) slices of M x N fp32) in the same time unit.
  const bool pair_t = gemm_use_pair(M);
  const int64_t tiles = pair_t ? ((M + 255) / 256) * ((N + 255) / 256) : ((M + 127) / 128) * ((N + 255) / 256);
  const int64_t slots = pair_t ? num_sms() / 2 : num_sms();
  const int64_t nkb = (K + 63) / 64;
  if (epi == EPI_F32 && batch == 1 && nkb >= 16 && ldo == N) {
    // one k-block of one tile ~ 0.35 us; the reduction streams (s + 2) M N 4 bytes at ~6 TB/s
    auto cost = [&](int64_t sp) {
      const int64_t kps_ = (nkb + sp - 1) / sp;
      const double waves = (double)((tiles * sp + slots - 1) / slots);
      const double red = sp > 1 ? (double)(sp + 2) * M * N * 4 / 6.0e6 / 0.35 : 0.0;
      return waves * (double)kps_ + red;
    };
    int splits = 1;
    for (int64_t sp = 2; sp <= std::min<int64_t>(16, nkb / 8); ++sp)
      if (cost(sp) < 0.93 * cost(splits)) splits = (int)sp;
    const int kps = (int)((nkb + splits - 1) / splits);
    splits = (int)((nkb + kps - 1) / kps);
    if (splits > 1) {
      at::Tensor ws = at::empty({(int64_t)splits * M * N}, out.options().dtype(at::kFloat));
      g.out = ws.data_ptr();
      g.ldo = N;
      g.out_bs = M * N;
      g.accumulate = 0;
      g.k_splits = splits;
      g.kb_per_split = kps;
      gemm_launch(g, stream);
      NG_TRACE("[gemm]   split-K reduce splits=%d n=%lld\n", splits, (long long)(M * N));
      splitk_reduce(ws.data_ptr<float>(), splits, M * N, out.data_ptr<float>(), accumulate, stream);
      NG_TRACE("[gemm]   reduce launched\n");
      return;
    }
  }
  gemm_launch(g, stream);
}

}  // namespace ng
