// RMSNorm + adaLN modulation (forward/backward) and the head's LayerNorm, for sm_100a.
//
// Forward: one warp per row, the row held in registers (C <= 2048, C % 8 == 0), 16-byte loads.
// Backward: one CTA per chunk of <= 64 rows of one modulation group. Phase 1 (a warp per row) computes the row's
// mean(dxn * xn); phase 2 (a thread per 8 columns) writes dx and keeps per-column partial sums of d_shift, d_scale and
// d_w in registers, stored per chunk. A second kernel reduces the chunk partials in a fixed order (deterministic).
// Reference math: baselines/PixelGen/src/models/layers/rmsnorm.py:5-20, JiT_T2I.py:75-76 (modulate),
// baselines/PixelGen/src/models/layers/fused_norm.py:64-140 (the same fused sums, Triton).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "finish.cuh"
#include "reduce.h"
#include "status.h"

namespace ng {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  f[0] = bf16_bits_lo(u.x);
  f[1] = bf16_bits_hi(u.x);
  f[2] = bf16_bits_lo(u.y);
  f[3] = bf16_bits_hi(u.y);
  f[4] = bf16_bits_lo(u.z);
  f[5] = bf16_bits_hi(u.z);
  f[6] = bf16_bits_lo(u.w);
  f[7] = bf16_bits_hi(u.w);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]);
  u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]);
  u.w = pack_bf16(f[6], f[7]);
  return u;
}

__device__ __forceinline__ void load_w8(const float* w, int c, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(w + c));
  const float4 b = __ldg(reinterpret_cast<const float4*>(w + c + 4));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = a.z;
  f[3] = a.w;
  f[4] = b.x;
  f[5] = b.y;
  f[6] = b.z;
  f[7] = b.w;
}

constexpr int MAXV = 8;  // 16-byte vectors per lane: C <= 32 * 8 * 8 = 2048

template <bool MOD, bool MXO = false>
__global__ void __launch_bounds__(256) rms_mod_fwd_kernel(const bf16* __restrict__ x, const float* __restrict__ w,
                                                          const bf16* __restrict__ shift, int64_t ld_sh,
                                                          const bf16* __restrict__ scale, int64_t ld_sc,
                                                          bf16* __restrict__ h, float* __restrict__ rstd, int M, int C,
                                                          int rpg, float eps, uint8_t* __restrict__ q = nullptr,
                                                          uint8_t* __restrict__ sf = nullptr,
                                                          const int* __restrict__ seg = nullptr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= M) return;
  const int nv = C >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * C);
  uint4 xv[MAXV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      xv[i] = xr[v];
      float f[8];
      unpack8(xv[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)C + eps);
  if (lane == 0) rstd[row] = r;
  const int g = seg != nullptr ? seg[row] : row / rpg;  // packed rows: the row's sample from the segment table
  uint4* hr = reinterpret_cast<uint4*>(h + (int64_t)row * C);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    uint4 pk = make_uint4(0u, 0u, 0u, 0u);
    if (v < nv) {
      float f[8], wf[8];
      unpack8(xv[i], f);
      load_w8(w, v * 8, wf);
      if (MOD) {
        float sh[8], sc[8];
        unpack8(*reinterpret_cast<const uint4*>(shift + (int64_t)g * ld_sh + v * 8), sh);
        unpack8(*reinterpret_cast<const uint4*>(scale + (int64_t)g * ld_sc + v * 8), sc);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = wf[j] * (f[j] * r) * (1.f + sc[j]) + sh[j];
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = wf[j] * (f[j] * r);
      }
      pk = pack8(f);
      hr[v] = pk;
    }
    if (MXO) {
      // MXFP8 copy of h (the input of the next MX GEMM): a 32-value block is the 8-value vectors of 4 adjacent lanes;
      // the values are the bf16-rounded h, so q and the scales equal a separate quantization of h
      float hv[8];
      float am = 0.f;
      if (v < nv) {
        unpack8(pk, hv);
#pragma unroll
        for (int j = 0; j < 8; ++j) am = fmaxf(am, fabsf(hv[j]));
      }
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
      if (v < nv) {
        const int e = mx_scale_exp(am);
        const float inv = ldexpf(1.f, -e);
        uint2 o;
        o.x = e4m3x4(hv[0] * inv, hv[1] * inv, hv[2] * inv, hv[3] * inv);
        o.y = e4m3x4(hv[4] * inv, hv[5] * inv, hv[6] * inv, hv[7] * inv);
        *reinterpret_cast<uint2*>(q + (int64_t)row * C + v * 8) = o;
        if ((v & 3) == 0) sf[mx_sf_offset(row, v >> 2, C / 128)] = (uint8_t)(e + 127);
      }
    }
  }
}

constexpr int BWD_ROWS = 64;

// Grid: (chunks_per_group, G). Partials: part[chunk_id][3][C], chunk_id = g * chunks_per_group + chunk.
template <bool MOD>
__global__ void __launch_bounds__(256) rms_mod_bwd_kernel(const bf16* __restrict__ dh, const bf16* __restrict__ x,
                                                          const float* __restrict__ rstd, const float* __restrict__ w,
                                                          const bf16* __restrict__ scale, int64_t ld_sc,
                                                          const bf16* __restrict__ dres, bf16* __restrict__ dx,
                                                          float* __restrict__ part, int M, int C, int rpg,
                                                          const int* __restrict__ cu = nullptr,
                                                          FinishArgs fa = FinishArgs{}) {
  __shared__ float s_c[BWD_ROWS];
  const int g = blockIdx.y, chunk = blockIdx.x;
  // rows of group g: [g rpg, (g + 1) rpg), or [cu[g], cu[g + 1]) for packed rows; a chunk past its group's end writes
  // zero partials
  const int gb = cu != nullptr ? cu[g] : g * rpg;
  const int ge = cu != nullptr ? cu[g + 1] : min(g * rpg + rpg, M);
  const int r0 = gb + chunk * BWD_ROWS;
  const int r1 = min(ge, r0 + BWD_ROWS);
  const int nrows = r1 - r0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = C >> 3;
  // ---- phase 1: per-row mean(dxn * xn), a warp per row
  for (int rr = warp; rr < nrows; rr += 8) {
    const int row = r0 + rr;
    const uint4* dr = reinterpret_cast<const uint4*>(dh + (int64_t)row * C);
    const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * C);
    const float r = rstd[row];
    float acc = 0.f;
    for (int v = lane; v < nv; v += 32) {
      float d[8], xf[8], wf[8];
      unpack8(dr[v], d);
      unpack8(xr[v], xf);
      load_w8(w, v * 8, wf);
      if (MOD) {
        float sc[8];
        unpack8(*reinterpret_cast<const uint4*>(scale + (int64_t)g * ld_sc + v * 8), sc);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc += d[j] * (1.f + sc[j]) * wf[j] * xf[j] * r;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc += d[j] * wf[j] * xf[j] * r;
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) s_c[rr] = acc / (float)C;
  }
  __syncthreads();
  // ---- phase 2: a thread per 8 columns walks the chunk's rows
  const int v = threadIdx.x;
  if (v < nv) {
    const int c0 = v * 8;
    float wf[8], sc[8];
    load_w8(w, c0, wf);
    if (MOD) {
      unpack8(*reinterpret_cast<const uint4*>(scale + (int64_t)g * ld_sc + c0), sc);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) sc[j] = 0.f;
    }
    float psh[8], psc[8], pw[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) psh[j] = psc[j] = pw[j] = 0.f;
    for (int rr = 0; rr < nrows; ++rr) {
      const int row = r0 + rr;
      const float r = rstd[row];
      const float cm = s_c[rr];
      float d[8], xf[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(dh + (int64_t)row * C + c0), d);
      unpack8(*reinterpret_cast<const uint4*>(x + (int64_t)row * C + c0), xf);
      float rs[8];
      if (dres != nullptr) {
        unpack8(*reinterpret_cast<const uint4*>(dres + (int64_t)row * C + c0), rs);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) rs[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xn = xf[j] * r;
        const float u = wf[j] * xn;
        const float du = d[j] * (1.f + sc[j]);
        psh[j] += d[j];
        psc[j] += d[j] * u;
        pw[j] += du * xn;
        const float dxn = du * wf[j];
        o[j] = r * (dxn - xn * cm) + rs[j];
      }
      *reinterpret_cast<uint4*>(dx + (int64_t)row * C + c0) = pack8(o);
    }
    const int cid = g * gridDim.x + chunk;
    float* pp = part + (int64_t)cid * 3 * C;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      pp[c0 + j] = psh[j];
      pp[C + c0 + j] = psc[j];
      pp[2 * C + c0 + j] = pw[j];
    }
  }
  if (fa.cnt != nullptr) finish_partials<3>(part, 3 * C, C, gridDim.x, g, fa);
}

// Bandwidth-shaped variant for C = 256 * VPL (the ladder widths 768 .. 1792). Phase 1: a warp per row, lane l owning
// columns 8 (l + 32 k), k < VPL: dh, x, dres are read once, the row's mean(dxn * xn) reduced in the warp and dx written
// at once. Phase 2: the column sums for d_shift, d_scale, d_w over the chunk's rows (dh and x again, now from L2), all
// 256 threads busy: G2 groups of C / 8 threads take alternate rows and are added up in shared memory.
template <bool MOD, int VPL>
__global__ void __launch_bounds__(256, VPL <= 4 ? 2 : 1) rms_mod_bwd_kernel2(const bf16* __restrict__ dh, const bf16* __restrict__ x,
                                                           const float* __restrict__ rstd, const float* __restrict__ w,
                                                           const bf16* __restrict__ scale, int64_t ld_sc,
                                                           const bf16* __restrict__ dres, bf16* __restrict__ dx,
                                                           float* __restrict__ part, int M, int rpg,
                                                           const int* __restrict__ cu = nullptr,
                                                           FinishArgs fa = FinishArgs{}) {
  constexpr int C = 256 * VPL, NV = C / 8;
  constexpr int G2 = 256 / NV;  // row groups in phase 2
  __shared__ float red[G2 > 1 ? (G2 - 1) * 3 * C : 1];
  const int g = blockIdx.y, chunk = blockIdx.x;
  const int gb = cu != nullptr ? cu[g] : g * rpg;  // as in rms_mod_bwd_kernel
  const int ge = cu != nullptr ? cu[g + 1] : min(g * rpg + rpg, M);
  const int r0 = gb + chunk * BWD_ROWS;
  const int r1 = min(ge, r0 + BWD_ROWS);
  const int nrows = r1 - r0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bf16* sc_row = MOD ? scale + (int64_t)g * ld_sc : nullptr;
  // ---- phase 1
  for (int rr = warp; rr < nrows; rr += 8) {
    const int64_t row = r0 + rr;
    const float r = rstd[row];
    uint4 dv[VPL], xv[VPL];
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int v = lane + 32 * k;
      dv[k] = reinterpret_cast<const uint4*>(dh + row * C)[v];
      xv[k] = reinterpret_cast<const uint4*>(x + row * C)[v];
    }
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int c0 = 8 * (lane + 32 * k);
      float d[8], xf[8], wf[8], sc[8];
      unpack8(dv[k], d);
      unpack8(xv[k], xf);
      load_w8(w, c0, wf);
      if (MOD) {
        unpack8(__ldg(reinterpret_cast<const uint4*>(sc_row + c0)), sc);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) sc[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) acc += d[j] * (1.f + sc[j]) * wf[j] * xf[j] * r;
    }
    const float cm = warp_sum(acc) / (float)C;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int c0 = 8 * (lane + 32 * k);
      float d[8], xf[8], wf[8], sc[8], rs[8], o[8];
      unpack8(dv[k], d);
      unpack8(xv[k], xf);
      // the residual gradient is read only here (not held across the row sum: fewer registers, two CTAs per SM)
      unpack8(dres != nullptr ? reinterpret_cast<const uint4*>(dres + row * C)[lane + 32 * k] : make_uint4(0, 0, 0, 0),
              rs);
      load_w8(w, c0, wf);
      if (MOD) {
        unpack8(__ldg(reinterpret_cast<const uint4*>(sc_row + c0)), sc);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) sc[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xn = xf[j] * r;
        o[j] = r * (d[j] * (1.f + sc[j]) * wf[j] - xn * cm) + rs[j];
      }
      reinterpret_cast<uint4*>(dx + row * C)[lane + 32 * k] = pack8(o);
    }
  }
  // ---- phase 2
  const int v = threadIdx.x % NV, grp = threadIdx.x / NV;
  const bool active = grp < G2;
  const int c0 = v * 8;
  float wf[8], sc[8];
  float psh[8], psc[8], pw[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) psh[j] = psc[j] = pw[j] = 0.f;
  if (active) {
    load_w8(w, c0, wf);
    if (MOD) {
      unpack8(__ldg(reinterpret_cast<const uint4*>(sc_row + c0)), sc);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) sc[j] = 0.f;
    }
    // the loads of four rows are issued before their math (the chunk's rows come back from L2: latency, not
    // bandwidth, bounds this loop); the rows are still added in the order rr, rr + G2, ...
    for (int rr = grp; rr < nrows; rr += 4 * G2) {
      uint4 dv[4], xv[4];
      float rv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = rr + u * G2;
        if (q < nrows) {
          const int64_t row = r0 + q;
          rv[u] = rstd[row];
          dv[u] = *reinterpret_cast<const uint4*>(dh + row * C + c0);
          xv[u] = *reinterpret_cast<const uint4*>(x + row * C + c0);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (rr + u * G2 < nrows) {
          float d[8], xf[8];
          unpack8(dv[u], d);
          unpack8(xv[u], xf);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xn = xf[j] * rv[u];
            psh[j] += d[j];
            psc[j] += d[j] * wf[j] * xn;
            pw[j] += d[j] * (1.f + sc[j]) * xn;
          }
        }
      }
    }
  }
  bool writer = active;
  if (G2 > 1) {
    if (active && grp > 0) {
      float* dst = red + (grp - 1) * 3 * C;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        dst[c0 + j] = psh[j];
        dst[C + c0 + j] = psc[j];
        dst[2 * C + c0 + j] = pw[j];
      }
    }
    __syncthreads();
    writer = grp == 0;
    if (writer) {
      for (int q = 0; q < G2 - 1; ++q) {
        const float* src = red + q * 3 * C;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          psh[j] += src[c0 + j];
          psc[j] += src[C + c0 + j];
          pw[j] += src[2 * C + c0 + j];
        }
      }
    }
  }
  if (writer) {
    const int cid = g * gridDim.x + chunk;
    float* pp = part + (int64_t)cid * 3 * C;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      pp[c0 + j] = psh[j];
      pp[C + c0 + j] = psc[j];
      pp[2 * C + c0 + j] = pw[j];
    }
  }
  // the group's last CTA adds the group's chunks in a fixed order: no group-sum launches
  if (fa.cnt != nullptr) finish_partials<3>(part, 3 * C, C, gridDim.x, g, fa);
}

// Reduction of the chunk partials for the no-allocation entry point, in two launches that allocate nothing.
// Stage 1, grid (ceil(C / 256), G): one thread per (column, group) adds the group's chunk partials in chunk order and
// writes d_shift / d_scale (strided fp32 views, may be null) and the group's d_w partial into gw [G, C].
__global__ void rms_mod_bwd_group_reduce(const float* __restrict__ part, int chunks, int C, float* dshift,
                                         int64_t ld_dsh, float* dscale, int64_t ld_dsc, float* __restrict__ gw) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x, g = blockIdx.y;
  if (c >= C) return;
  float a = 0.f, b = 0.f, t = 0.f;
  for (int k = 0; k < chunks; ++k) {
    const float* pp = part + (int64_t)(g * chunks + k) * 3 * C;
    a += pp[c];
    b += pp[C + c];
    t += pp[2 * C + c];
  }
  if (dshift != nullptr) dshift[(int64_t)g * ld_dsh + c] = a;
  if (dscale != nullptr) dscale[(int64_t)g * ld_dsc + c] = b;
  gw[(int64_t)g * C + c] = t;
}

// Stage 2: d_w[c] += sum over groups of gw[g, c], four independent accumulators (groups g = 4i + j) combined in a
// fixed order, so the result is the same on every run.
__global__ void rms_mod_bwd_dw_reduce(const float* __restrict__ gw, int G, int C, float* __restrict__ dw) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float t[4] = {0.f, 0.f, 0.f, 0.f};
  int g = 0;
  for (; g + 4 <= G; g += 4)
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] += gw[(int64_t)(g + j) * C + c];
  for (int j = 0; g < G; ++g, ++j) t[j] += gw[(int64_t)g * C + c];
  dw[c] += (t[0] + t[1]) + (t[2] + t[3]);
}

// ------------------------------------------------------------------------------------------------------- LayerNorm
__global__ void __launch_bounds__(256) layernorm_fwd_kernel(const bf16* __restrict__ x, bf16* __restrict__ h,
                                                            float* __restrict__ mu_out, float* __restrict__ rstd_out,
                                                            int M, int C, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= M) return;
  const int nv = C >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * C);
  uint4 xv[MAXV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      xv[i] = xr[v];
      float f[8];
      unpack8(xv[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += f[j];
    }
  }
  const float mu = warp_sum(s) / (float)C;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      float f[8];
      unpack8(xv[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += (f[j] - mu) * (f[j] - mu);
    }
  }
  const float r = rsqrtf(warp_sum(ss) / (float)C + eps);
  if (lane == 0) {
    mu_out[row] = mu;
    rstd_out[row] = r;
  }
  uint4* hr = reinterpret_cast<uint4*>(h + (int64_t)row * C);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      float f[8];
      unpack8(xv[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = (f[j] - mu) * r;
      hr[v] = pack8(f);
    }
  }
}

__global__ void __launch_bounds__(256) layernorm_bwd_kernel(const bf16* __restrict__ dh, const bf16* __restrict__ x,
                                                            const float* __restrict__ mu_in,
                                                            const float* __restrict__ rstd_in, bf16* __restrict__ dx,
                                                            int M, int C) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= M) return;
  const int nv = C >> 3;
  const float mu = mu_in[row], r = rstd_in[row];
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * C);
  const uint4* dr = reinterpret_cast<const uint4*>(dh + (int64_t)row * C);
  uint4 xv[MAXV], dv[MAXV];
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      xv[i] = xr[v];
      dv[i] = dr[v];
      float f[8], d[8];
      unpack8(xv[i], f);
      unpack8(dv[i], d);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s1 += d[j];
        s2 += d[j] * (f[j] - mu) * r;
      }
    }
  }
  const float m1 = warp_sum(s1) / (float)C, m2 = warp_sum(s2) / (float)C;
  uint4* out = reinterpret_cast<uint4*>(dx + (int64_t)row * C);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      float f[8], d[8];
      unpack8(xv[i], f);
      unpack8(dv[i], d);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = r * (d[j] - m1 - (f[j] - mu) * r * m2);
      out[v] = pack8(f);
    }
  }
}

// ====================================================================================================== torch glue
static const bf16* bptr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<const bf16*>(t->data_ptr()) : nullptr;
}
static int64_t ld_of(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->stride(0) : 0;
}

static void check_rows(const at::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous() && x.scalar_type() == at::kBFloat16,
              "contiguous 2-D bf16 CUDA tensor expected");
  TORCH_CHECK(x.size(1) % 8 == 0 && x.size(1) <= 2048, "norm kernels need C % 8 == 0 and C <= 2048");
}

void rms_mod_fwd(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& shift,
                 const c10::optional<at::Tensor>& scale, const at::Tensor& h, const at::Tensor& rstd, int64_t rpg,
                 double eps, const c10::optional<at::Tensor>& seg) {
  check_rows(x);
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous(), "fp32 weight expected");
  const at::cuda::CUDAGuard guard(x.device());
  const int M = x.size(0), C = x.size(1);
  auto s = at::cuda::getCurrentCUDAStream();
  const bool mod = scale.has_value() && scale->defined();
  const int* segp = nullptr;
  if (seg.has_value() && seg->defined()) {
    TORCH_CHECK(mod && seg->scalar_type() == at::kInt && seg->is_contiguous() && seg->numel() == M && seg->is_cuda(),
                "rms_mod_fwd: seg must be a [M] int32 CUDA tensor (modulated rows only)");
    segp = seg->data_ptr<int>();
  }
  dim3 grid((M + 7) / 8);
  if (mod)
    rms_mod_fwd_kernel<true><<<grid, 256, 0, s>>>(
        reinterpret_cast<const bf16*>(x.data_ptr()), w.data_ptr<float>(), bptr(shift), ld_of(shift), bptr(scale),
        ld_of(scale), reinterpret_cast<bf16*>(h.data_ptr()), rstd.data_ptr<float>(), M, C, (int)rpg, (float)eps,
        nullptr, nullptr, segp);
  else
    rms_mod_fwd_kernel<false><<<grid, 256, 0, s>>>(reinterpret_cast<const bf16*>(x.data_ptr()), w.data_ptr<float>(),
                                                   nullptr, 0, nullptr, 0, reinterpret_cast<bf16*>(h.data_ptr()),
                                                   rstd.data_ptr<float>(), M, C, (int)rpg, (float)eps);
  NG_LAUNCH_CHECK();
}

// rms_mod_fwd that also writes h's MXFP8 copy: q [M, C] e4m3, sf the scale blocks of csrc/mx.cu's layout (rows padded
// to a multiple of 256; padding rows are left as the caller filled them). C a multiple of 128.
void rms_mod_fwd_mx(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& shift,
                    const c10::optional<at::Tensor>& scale, const at::Tensor& h, const at::Tensor& rstd,
                    const at::Tensor& q, const at::Tensor& sf, int64_t rpg, double eps) {
  check_rows(x);
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous(), "fp32 weight expected");
  const int M = x.size(0), C = x.size(1);
  TORCH_CHECK(C % 128 == 0, "rms_mod_fwd_mx: C must be a multiple of 128");
  TORCH_CHECK(q.scalar_type() == at::kByte && q.is_contiguous() && q.numel() == (int64_t)M * C, "q: [M, C] uint8");
  TORCH_CHECK(sf.scalar_type() == at::kByte && sf.is_contiguous() &&
                  sf.numel() >= ((int64_t)M + 255) / 256 * 256 * (C / 32),
              "sf: scale blocks of [rows padded to 256, C / 32]");
  const at::cuda::CUDAGuard guard(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const bool mod = scale.has_value() && scale->defined();
  dim3 grid((M + 7) / 8);
  if (mod)
    rms_mod_fwd_kernel<true, true><<<grid, 256, 0, s>>>(
        reinterpret_cast<const bf16*>(x.data_ptr()), w.data_ptr<float>(), bptr(shift), ld_of(shift), bptr(scale),
        ld_of(scale), reinterpret_cast<bf16*>(h.data_ptr()), rstd.data_ptr<float>(), M, C, (int)rpg, (float)eps,
        q.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>());
  else
    rms_mod_fwd_kernel<false, true><<<grid, 256, 0, s>>>(
        reinterpret_cast<const bf16*>(x.data_ptr()), w.data_ptr<float>(), nullptr, 0, nullptr, 0,
        reinterpret_cast<bf16*>(h.data_ptr()), rstd.data_ptr<float>(), M, C, (int)rpg, (float)eps,
        q.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>());
  NG_LAUNCH_CHECK();
}

void rms_mod_bwd(const at::Tensor& dh, const at::Tensor& x, const at::Tensor& rstd, const at::Tensor& w,
                 const c10::optional<at::Tensor>& scale, const c10::optional<at::Tensor>& dres, const at::Tensor& dx,
                 const c10::optional<at::Tensor>& dw, const c10::optional<at::Tensor>& dshift,
                 const c10::optional<at::Tensor>& dscale, int64_t rpg, const c10::optional<at::Tensor>& cu,
                 int64_t max_rows) {
  check_rows(x);
  check_rows(dh);
  const at::cuda::CUDAGuard guard(x.device());
  const int M = x.size(0), C = x.size(1);
  const bool mod = scale.has_value() && scale->defined();
  // packed rows: group g is rows [cu[g], cu[g + 1]), every group at most max_rows long
  const bool packed = cu.has_value() && cu->defined();
  const int* cup = nullptr;
  if (packed) {
    TORCH_CHECK(mod && cu->scalar_type() == at::kInt && cu->is_contiguous() && cu->numel() >= 2 && cu->is_cuda() &&
                    max_rows > 0,
                "rms_mod_bwd: cu must be a [G + 1] int32 CUDA tensor of row offsets, with max_rows > 0");
    cup = cu->data_ptr<int>();
  }
  const int G = packed ? (int)cu->numel() - 1 : mod ? (M + (int)rpg - 1) / (int)rpg : 1;
  TORCH_CHECK(G <= 65535, "rms_mod_bwd: at most 65535 groups");
  const int rows_per_group = mod ? (int)rpg : M;
  const int chunks = ((packed ? (int)max_rows : rows_per_group) + BWD_ROWS - 1) / BWD_ROWS;
  auto s = at::cuda::getCurrentCUDAStream();
  // chunk partials, then the group rows of the d_w sums (the kernel's last CTA per group writes d_shift, d_scale and
  // the group's d_w row: no group-sum launches)
  at::Tensor part = at::empty({(int64_t)G * chunks * 3 * C + (int64_t)G * C}, x.options().dtype(at::kFloat));
  dim3 grid(chunks, G);
  FinishArgs fa{};
  fa.gout[0] = (mod && dshift.has_value() && dshift->defined()) ? dshift->data_ptr<float>() : nullptr;
  fa.gout[1] = (mod && dscale.has_value() && dscale->defined()) ? dscale->data_ptr<float>() : nullptr;
  fa.gld[0] = fa.gout[0] != nullptr ? ld_of(dshift) : 0;
  fa.gld[1] = fa.gout[1] != nullptr ? ld_of(dscale) : 0;
  fa.scratch = part.data_ptr<float>() + (int64_t)G * chunks * 3 * C;
  // a group of many chunks (the plain norm over all rows) would make its last CTA a long serial tail: then the host's
  // two-stage reductions take the partials instead
  const bool in_kernel = chunks <= kFinishMaxChunks;
  fa.cnt = in_kernel ? finish_counters(s, G) : nullptr;
  const bf16* scp = mod ? bptr(scale) : nullptr;
  const int64_t ldsc = mod ? ld_of(scale) : 0;
  bool done = true;
#define NG_RMS_BWD2(V)                                                                                               \
  if (mod)                                                                                                           \
    rms_mod_bwd_kernel2<true, V><<<grid, 256, 0, s>>>(                                                              \
        reinterpret_cast<const bf16*>(dh.data_ptr()), reinterpret_cast<const bf16*>(x.data_ptr()),                   \
        rstd.data_ptr<float>(), w.data_ptr<float>(), scp, ldsc, bptr(dres), reinterpret_cast<bf16*>(dx.data_ptr()), \
        part.data_ptr<float>(), M, rows_per_group, cup, fa);                                                         \
  else                                                                                                               \
    rms_mod_bwd_kernel2<false, V><<<grid, 256, 0, s>>>(                                                             \
        reinterpret_cast<const bf16*>(dh.data_ptr()), reinterpret_cast<const bf16*>(x.data_ptr()),                   \
        rstd.data_ptr<float>(), w.data_ptr<float>(), nullptr, 0, bptr(dres), reinterpret_cast<bf16*>(dx.data_ptr()), \
        part.data_ptr<float>(), M, rows_per_group, nullptr, fa);
  switch (C) {
    case 768: NG_RMS_BWD2(3) break;
    case 1024: NG_RMS_BWD2(4) break;
    case 1280: NG_RMS_BWD2(5) break;
    case 1536: NG_RMS_BWD2(6) break;
    case 1792: NG_RMS_BWD2(7) break;
    default: done = false;
  }
#undef NG_RMS_BWD2
  if (done) {
  } else if (mod)
    rms_mod_bwd_kernel<true><<<grid, 256, 0, s>>>(
        reinterpret_cast<const bf16*>(dh.data_ptr()), reinterpret_cast<const bf16*>(x.data_ptr()),
        rstd.data_ptr<float>(), w.data_ptr<float>(), bptr(scale), ld_of(scale), bptr(dres),
        reinterpret_cast<bf16*>(dx.data_ptr()), part.data_ptr<float>(), M, C, rows_per_group, cup, fa);
  else
    rms_mod_bwd_kernel<false><<<grid, 256, 0, s>>>(
        reinterpret_cast<const bf16*>(dh.data_ptr()), reinterpret_cast<const bf16*>(x.data_ptr()),
        rstd.data_ptr<float>(), w.data_ptr<float>(), nullptr, 0, bptr(dres), reinterpret_cast<bf16*>(dx.data_ptr()),
        part.data_ptr<float>(), M, C, rows_per_group, nullptr, fa);
  NG_LAUNCH_CHECK();
  float* dwp = (dw.has_value() && dw->defined()) ? dw->data_ptr<float>() : nullptr;
  if (in_kernel) {  // d_w: the column sums of the G group rows the kernel left in the scratch
    if (dwp != nullptr) colsum_launch(fa.scratch, false, G, C, C, dwp, true, s);
    return;
  }
  const float* pp = part.data_ptr<float>();
  if (mod) {
    group_sum_launch(pp, G, chunks, C, 3 * C, fa.gout[0], fa.gld[0], s);
    group_sum_launch(pp + C, G, chunks, C, 3 * C, fa.gout[1], fa.gld[1], s);
  }
  if (dwp != nullptr) colsum_launch(pp + 2 * C, false, (int64_t)G * chunks, C, 3 * C, dwp, true, s);
}

void layernorm_fwd(const at::Tensor& x, const at::Tensor& h, const at::Tensor& mu, const at::Tensor& rstd, double eps) {
  check_rows(x);
  const at::cuda::CUDAGuard guard(x.device());
  const int M = x.size(0), C = x.size(1);
  layernorm_fwd_kernel<<<(M + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), reinterpret_cast<bf16*>(h.data_ptr()), mu.data_ptr<float>(),
      rstd.data_ptr<float>(), M, C, (float)eps);
  NG_LAUNCH_CHECK();
}

void layernorm_bwd(const at::Tensor& dh, const at::Tensor& x, const at::Tensor& mu, const at::Tensor& rstd,
                   const at::Tensor& dx) {
  check_rows(x);
  const at::cuda::CUDAGuard guard(x.device());
  const int M = x.size(0), C = x.size(1);
  layernorm_bwd_kernel<<<(M + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(dh.data_ptr()), reinterpret_cast<const bf16*>(x.data_ptr()), mu.data_ptr<float>(),
      rstd.data_ptr<float>(), reinterpret_cast<bf16*>(dx.data_ptr()), M, C);
  NG_LAUNCH_CHECK();
}

}  // namespace ng

// =============================================================================================== no-allocation entry
// ng_rms_mod_bwd_noalloc (declared and documented in csrc/noalloc.h): the same two kernels as rms_mod_bwd, with the
// chunk partials in a fixed device array instead of a PyTorch allocation. This block adds a path; it changes none.
#include <mutex>

#include "noalloc.h"

namespace ng {
namespace {
// The scratch: fp32 partial column sums, [chunks * groups][3][C]. Host code must not use this name as an address.
static __device__ __align__(256) float g_noalloc_rms_scratch[NG_NOALLOC_RMS_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
constexpr int kMaxGridY = 65535;  // the groups are the second grid dimension of the launches
std::mutex g_noalloc_mu;
float* g_noalloc_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array for the current device, looked up once per device.
float* noalloc_scratch(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = NG_NOALLOC_ERR_SETUP;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_rms_scratch) != cudaSuccess || p == nullptr) {
      *err = NG_NOALLOC_ERR_SETUP;
      return nullptr;
    }
    g_noalloc_addr[dev] = static_cast<float*>(p);
  }
  return g_noalloc_addr[dev];
}
}  // namespace
}  // namespace ng

extern "C" __attribute__((visibility("default"))) int ng_rms_mod_bwd_noalloc(
    const void* dh, const void* x, const float* rstd, const float* w, const void* scale, int64_t ld_scale,
    const void* dres, void* dx, float* dw, float* dshift, int64_t ld_dshift, float* dscale, int64_t ld_dscale, int M,
    int C, int rows_per_group, cudaStream_t stream) {
  using namespace ng;
  if (dh == nullptr || x == nullptr || rstd == nullptr || w == nullptr || dx == nullptr || M <= 0 || C <= 0 ||
      C % 8 != 0 || C > 2048 || (scale != nullptr && rows_per_group <= 0))
    return NG_NOALLOC_ERR_ARGS;
  const bool mod = scale != nullptr;
  const int rpg = mod ? rows_per_group : M;
  const int G = mod ? (M + rpg - 1) / rpg : 1;
  const int chunks = (rpg + BWD_ROWS - 1) / BWD_ROWS;
  if (G > kMaxGridY) return NG_NOALLOC_ERR_ARGS;
  const int64_t need = (int64_t)G * chunks * 3 * C + (int64_t)G * C;  // chunk partials + per-group d_w partials
  if (need > (int64_t)NG_NOALLOC_RMS_SCRATCH_FLOATS) return NG_NOALLOC_ERR_TOO_LARGE;
  int err = NG_NOALLOC_OK;
  float* part = noalloc_scratch(&err);
  if (part == nullptr) return err;
  // An error left by earlier work on this thread belongs to its owner: leave it in place and launch nothing, so the
  // launch checks below only ever see this call's own errors.
  if (cudaPeekAtLastError() != cudaSuccess) return NG_NOALLOC_ERR_PENDING;
  const dim3 grid(chunks, G);
  const bf16* sc = static_cast<const bf16*>(scale);
  if (mod)
    rms_mod_bwd_kernel<true><<<grid, 256, 0, stream>>>(static_cast<const bf16*>(dh), static_cast<const bf16*>(x), rstd,
                                                       w, sc, ld_scale, static_cast<const bf16*>(dres),
                                                       static_cast<bf16*>(dx), part, M, C, rpg);
  else
    rms_mod_bwd_kernel<false><<<grid, 256, 0, stream>>>(static_cast<const bf16*>(dh), static_cast<const bf16*>(x),
                                                        rstd, w, nullptr, 0, static_cast<const bf16*>(dres),
                                                        static_cast<bf16*>(dx), part, M, C, rpg);
  if (cudaGetLastError() != cudaSuccess) return NG_NOALLOC_ERR_LAUNCH;
  float* gw = part + (int64_t)G * chunks * 3 * C;
  rms_mod_bwd_group_reduce<<<dim3((C + 255) / 256, G), 256, 0, stream>>>(
      part, chunks, C, mod ? dshift : nullptr, ld_dshift, mod ? dscale : nullptr, ld_dscale, gw);
  if (cudaGetLastError() != cudaSuccess) return NG_NOALLOC_ERR_LAUNCH;
  if (dw != nullptr) {
    rms_mod_bwd_dw_reduce<<<(C + 255) / 256, 256, 0, stream>>>(gw, G, C, dw);
    if (cudaGetLastError() != cudaSuccess) return NG_NOALLOC_ERR_LAUNCH;
  }
  return NG_NOALLOC_OK;
}

extern "C" __attribute__((visibility("default"))) const char* ng_noalloc_error_string(int code) {
  switch (code) {
    case NG_NOALLOC_OK: return "ok";
    case NG_NOALLOC_ERR_TOO_LARGE:
      return "ng_rms_mod_bwd_noalloc: the call needs more than NG_NOALLOC_RMS_SCRATCH_FLOATS (2097152) fp32 scratch "
             "values (ceil(rows_per_group / 64) * groups * 3 * C + groups * C); use the allocating entry point for it";
    case NG_NOALLOC_ERR_ARGS:
      return "ng_rms_mod_bwd_noalloc: bad arguments (null pointer, C % 8 != 0, C > 2048, a size <= 0, or more than "
             "65535 groups)";
    case NG_NOALLOC_ERR_PENDING:
      return "ng_rms_mod_bwd_noalloc: a CUDA error from earlier work is pending on this thread (cudaPeekAtLastError); "
             "nothing was launched and the error was left in place";
    case NG_NOALLOC_ERR_SETUP: return "ng_rms_mod_bwd_noalloc: could not resolve the scratch array on this device";
    case NG_NOALLOC_ERR_LAUNCH: return "ng_rms_mod_bwd_noalloc: kernel launch failed";
    default: return "ng_rms_mod_bwd_noalloc: unknown error code";
  }
}
