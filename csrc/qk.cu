// Per-head RMSNorm of q/k with the 2D RoPE fused in, forward and backward (head dim 64), for sm_100a.
// Forward: four lanes per (row, head) (qk_norm_fwd4_kernel): each lane keeps 16 of the head's 64 values, the head's
// sums take two shuffles. Backward: eight lanes per (row, head), two units in flight (qk_norm_bwd8_kernel). The
// one-thread-per-head kernels that come first are kept as the simplest statement of the math.
// Reference: q_norm/k_norm + apply_rotary_emb_real (baselines/PixelGen/src/models/transformer/JiT_T2I.py:141-166,
// baselines/PixelGen/src/models/layers/rope.py:53-69), the Triton lever K2 (fused_qk.py:55-200).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "reduce.h"
#include "status.h"

namespace ng {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void ld64(const bf16* p, float (&f)[64]) {
  const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 u = p4[i];
    f[8 * i + 0] = bf16_bits_lo(u.x);
    f[8 * i + 1] = bf16_bits_hi(u.x);
    f[8 * i + 2] = bf16_bits_lo(u.y);
    f[8 * i + 3] = bf16_bits_hi(u.y);
    f[8 * i + 4] = bf16_bits_lo(u.z);
    f[8 * i + 5] = bf16_bits_hi(u.z);
    f[8 * i + 6] = bf16_bits_lo(u.w);
    f[8 * i + 7] = bf16_bits_hi(u.w);
  }
}

__device__ __forceinline__ void st64(bf16* p, const float (&f)[64]) {
  uint4* p4 = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint4 u;
    u.x = pack_bf16(f[8 * i + 0], f[8 * i + 1]);
    u.y = pack_bf16(f[8 * i + 2], f[8 * i + 3]);
    u.z = pack_bf16(f[8 * i + 4], f[8 * i + 5]);
    u.w = pack_bf16(f[8 * i + 6], f[8 * i + 7]);
    p4[i] = u;
  }
}

template <bool ROPE>
__global__ void __launch_bounds__(256) qk_norm_fwd_kernel(const bf16* __restrict__ src, int64_t ld_src,
                                                          const float* __restrict__ w, const float* __restrict__ cosT,
                                                          const float* __restrict__ sinT, bf16* __restrict__ out,
                                                          float* __restrict__ rstd, int rows, int H, int L,
                                                          float eps) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (int64_t)rows * H) return;
  const int row = (int)(t / H), h = (int)(t - (int64_t)row * H);
  float x[64];
  ld64(src + row * ld_src + h * 64, x);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) ss += x[i] * x[i];
  const float r = rsqrtf(ss * (1.f / 64.f) + eps);
  rstd[t] = r;
#pragma unroll
  for (int i = 0; i < 64; ++i) x[i] = __ldg(w + i) * x[i] * r;
  if (ROPE) {
    const int pos = row % L;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float c = __ldg(cosT + pos * 32 + j), s = __ldg(sinT + pos * 32 + j);
      const float a = x[2 * j], b = x[2 * j + 1];
      x[2 * j] = a * c - b * s;
      x[2 * j + 1] = a * s + b * c;
    }
  }
  st64(out + (int64_t)row * H * 64 + h * 64, x);
}

// dw partials: part[block][64] (fixed-order reduction afterwards)
template <bool ROPE>
__global__ void __launch_bounds__(256) qk_norm_bwd_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ src,
                                                          int64_t ld_src, const float* __restrict__ rstd,
                                                          const float* __restrict__ w, const float* __restrict__ cosT,
                                                          const float* __restrict__ sinT, bf16* __restrict__ dsrc,
                                                          int64_t ld_dsrc, float* __restrict__ part, int rows, int H,
                                                          int L) {
  __shared__ float s_part[8][64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float dw[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) dw[i] = 0.f;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < (int64_t)rows * H;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(t / H), h = (int)(t - (int64_t)row * H);
    float d[64], x[64];
    ld64(dout + (int64_t)row * H * 64 + h * 64, d);
    ld64(src + row * ld_src + h * 64, x);
    if (ROPE) {
      const int pos = row % L;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float c = __ldg(cosT + pos * 32 + j), s = __ldg(sinT + pos * 32 + j);
        const float a = d[2 * j], b = d[2 * j + 1];
        d[2 * j] = a * c + b * s;
        d[2 * j + 1] = -a * s + b * c;
      }
    }
    const float r = rstd[t];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const float xh = x[i] * r;
      dw[i] += d[i] * xh;
      d[i] = d[i] * __ldg(w + i);  // d(xhat)
      dot += d[i] * xh;
    }
    dot *= (1.f / 64.f);
#pragma unroll
    for (int i = 0; i < 64; ++i) x[i] = r * (d[i] - x[i] * r * dot);
    st64(dsrc + row * ld_dsrc + h * 64, x);
  }
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    const float v = warp_sum(dw[i]);
    if (lane == 0) s_part[warp][i] = v;
  }
  __syncthreads();
  if (threadIdx.x < 64) {
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) a += s_part[k][threadIdx.x];
    part[(int64_t)blockIdx.x * 64 + threadIdx.x] = a;
  }
}

__global__ void reduce_cols_kernel(const float* __restrict__ part, int nparts, int C, float* __restrict__ acc) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float a = 0.f;
  for (int k = 0; k < nparts; ++k) a += part[(int64_t)k * C + c];
  acc[c] += a;
}

// ---------------------------------------------------------------------------------- four lanes per head (default)
// Lane q of a quad owns the 16-byte chunks q and q + 4 of the head (elements 8q..8q+7 and 8q+32..8q+39): for each of
// the two loads the quad reads 64 contiguous bytes. The head's sums are completed with two shuffles; the norm weight
// and the RoPE tables are read as float4.
__device__ __forceinline__ void ld8(const bf16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  f[0] = bf16_bits_lo(u.x);
  f[1] = bf16_bits_hi(u.x);
  f[2] = bf16_bits_lo(u.y);
  f[3] = bf16_bits_hi(u.y);
  f[4] = bf16_bits_lo(u.z);
  f[5] = bf16_bits_hi(u.z);
  f[6] = bf16_bits_lo(u.w);
  f[7] = bf16_bits_hi(u.w);
}
__device__ __forceinline__ void st8(bf16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]);
  u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]);
  u.w = pack_bf16(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void ldf8(const float* p, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x;
  f[1] = a.y;
  f[2] = a.z;
  f[3] = a.w;
  f[4] = b.x;
  f[5] = b.y;
  f[6] = b.z;
  f[7] = b.w;
}
__device__ __forceinline__ void ldf4(const float* p, float (&f)[4]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = a.z;
  f[3] = a.w;
}
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

template <bool ROPE>
__global__ void __launch_bounds__(256) qk_norm_fwd4_kernel(const bf16* __restrict__ src, int64_t ld_src,
                                                           const float* __restrict__ w, const float* __restrict__ cosT,
                                                           const float* __restrict__ sinT, bf16* __restrict__ out,
                                                           float* __restrict__ rstd, int rows, int H, int L,
                                                           float eps) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t unit = t >> 2;  // (row, head)
  const int q = threadIdx.x & 3;
  const bool valid = unit < (int64_t)rows * H;
  const int64_t u = valid ? unit : 0;
  const int row = (int)(u / H), h = (int)(u - (int64_t)row * H);
  const bf16* sp = src + row * ld_src + h * 64;
  float x[2][8];
  ld8(sp + 8 * q, x[0]);
  ld8(sp + 8 * q + 32, x[1]);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 2; ++k)
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x[k][i] * x[k][i];
  ss = quad_sum(ss);
  const float r = rsqrtf(ss * (1.f / 64.f) + eps);
  if (valid && q == 0) rstd[u] = r;
  const int pos = ROPE ? row % L : 0;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int e0 = 8 * q + 32 * k;
    float wf[8];
    ldf8(w + e0, wf);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[k][i] = wf[i] * x[k][i] * r;
    if (ROPE) {
      float c[4], sn[4];
      ldf4(cosT + pos * 32 + e0 / 2, c);
      ldf4(sinT + pos * 32 + e0 / 2, sn);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = x[k][2 * j], b = x[k][2 * j + 1];
        x[k][2 * j] = a * c[j] - b * sn[j];
        x[k][2 * j + 1] = a * sn[j] + b * c[j];
      }
    }
    if (valid) st8(out + (int64_t)row * H * 64 + h * 64 + e0, x[k]);
  }
}

// Backward with eight lanes per (row, head), one 16-byte vector of dout and of src per lane, two units in flight per
// lane (both units' loads are issued before either's math): few registers (four CTAs per SM) and many bytes in flight
// per thread, for the DRAM-bound image q/k backward; a dw partial row per block, summed in a fixed order afterwards.
template <bool ROPE>
__global__ void __launch_bounds__(256, 4) qk_norm_bwd8_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ src,
                                                              int64_t ld_src, const float* __restrict__ rstd,
                                                              const float* __restrict__ w, const float* __restrict__ cosT,
                                                              const float* __restrict__ sinT, bf16* __restrict__ dsrc,
                                                              int64_t ld_dsrc, float* __restrict__ part, int rows, int H,
                                                              int L) {
  __shared__ float s_part[8][64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, e = lane & 7;
  float dw[8], wf[8];
  ldf8(w + 8 * e, wf);
#pragma unroll
  for (int i = 0; i < 8; ++i) dw[i] = 0.f;
  const int64_t units = (int64_t)rows * H;
  const int64_t groups = ((int64_t)gridDim.x * blockDim.x) >> 3;
  const int64_t first = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
  // every group of eight runs the same number of iterations (its shuffles need all eight lanes)
  for (int64_t base = first; base - (threadIdx.x >> 3) < units; base += 2 * groups) {
    float d[2][8], x[2][8], r[2];
    int row[2], h[2];
    bool valid[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int64_t b = base + k * groups;
      valid[k] = b < units;
      const int64_t u = valid[k] ? b : 0;
      row[k] = (int)(u / H);
      h[k] = (int)(u - (int64_t)row[k] * H);
      ld8(dout + (int64_t)row[k] * H * 64 + h[k] * 64 + 8 * e, d[k]);
      ld8(src + row[k] * ld_src + h[k] * 64 + 8 * e, x[k]);
      r[k] = valid[k] ? rstd[u] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (ROPE) {
        const int pos = row[k] % L;
        float c[4], sn[4];
        ldf4(cosT + pos * 32 + 4 * e, c);
        ldf4(sinT + pos * 32 + 4 * e, sn);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = d[k][2 * j], bb = d[k][2 * j + 1];
          d[k][2 * j] = a * c[j] + bb * sn[j];
          d[k][2 * j + 1] = -a * sn[j] + bb * c[j];
        }
      }
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = x[k][i] * r[k];
        dw[i] += valid[k] ? d[k][i] * xh : 0.f;
        d[k][i] *= wf[i];  // d(xhat)
        dot += d[k][i] * xh;
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 4);
      dot *= 1.f / 64.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) x[k][i] = r[k] * (d[k][i] - x[k][i] * r[k] * dot);
      if (valid[k]) st8(dsrc + row[k] * ld_dsrc + h[k] * 64 + 8 * e, x[k]);
    }
  }
  // dw: lanes with the same e hold the same 8 columns; reduce over the 4 groups of the warp, then over warps
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float v = dw[i];
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    if (lane < 8) s_part[warp][8 * e + i] = v;
  }
  __syncthreads();
  if (threadIdx.x < 64) {
    float a = 0.f;
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) a += s_part[k2][threadIdx.x];
    part[(int64_t)blockIdx.x * 64 + threadIdx.x] = a;
  }
}

// ====================================================================================================== torch glue
static const float* fptr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr<float>() : nullptr;
}

void qk_norm_fwd(const at::Tensor& src, const at::Tensor& w, const c10::optional<at::Tensor>& cosT,
                 const c10::optional<at::Tensor>& sinT, const at::Tensor& out, const at::Tensor& rstd, int64_t L,
                 double eps) {
  TORCH_CHECK(src.is_cuda() && src.stride(1) == 1 && src.size(1) % 64 == 0, "qk_norm_fwd: bad source");
  TORCH_CHECK((src.stride(0) % 8) == 0 && (reinterpret_cast<uintptr_t>(src.data_ptr()) & 15) == 0,
              "qk_norm_fwd: 16-byte aligned rows expected");
  const at::cuda::CUDAGuard guard(src.device());
  const int rows = src.size(0), H = src.size(1) / 64;
  const int64_t n = (int64_t)rows * H;
  const int grid = (int)((4 * n + 255) / 256);  // four lanes per (row, head)
  auto s = at::cuda::getCurrentCUDAStream();
  const auto* sp = reinterpret_cast<const bf16*>(src.data_ptr());
  auto* op = reinterpret_cast<bf16*>(out.data_ptr());
  if (fptr(cosT) != nullptr)
    qk_norm_fwd4_kernel<true><<<grid, 256, 0, s>>>(sp, src.stride(0), w.data_ptr<float>(), fptr(cosT), fptr(sinT), op,
                                                   rstd.data_ptr<float>(), rows, H, (int)L, (float)eps);
  else
    qk_norm_fwd4_kernel<false><<<grid, 256, 0, s>>>(sp, src.stride(0), w.data_ptr<float>(), nullptr, nullptr, op,
                                                    rstd.data_ptr<float>(), rows, H, (int)L, (float)eps);
  NG_LAUNCH_CHECK();
}

void qk_norm_bwd(const at::Tensor& dout, const at::Tensor& src, const at::Tensor& rstd, const at::Tensor& w,
                 const c10::optional<at::Tensor>& cosT, const c10::optional<at::Tensor>& sinT, const at::Tensor& dsrc,
                 const c10::optional<at::Tensor>& dw, int64_t L) {
  TORCH_CHECK(src.is_cuda() && dout.is_contiguous() && dsrc.stride(1) == 1, "qk_norm_bwd: bad layout");
  const at::cuda::CUDAGuard guard(src.device());
  const int rows = src.size(0), H = src.size(1) / 64;
  const int64_t n = (int64_t)rows * H;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, src.get_device());
  // eight lanes per (row, head), two units per lane per iteration; four resident CTAs per SM
  const int grid = (int)std::min<int64_t>((8 * n + 255) / 256, 4 * (int64_t)sms);
  auto s = at::cuda::getCurrentCUDAStream();
  at::Tensor part = at::empty({(int64_t)grid * 64}, src.options().dtype(at::kFloat));
  const auto* dp = reinterpret_cast<const bf16*>(dout.data_ptr());
  const auto* sp = reinterpret_cast<const bf16*>(src.data_ptr());
  auto* op = reinterpret_cast<bf16*>(dsrc.data_ptr());
  if (fptr(cosT) != nullptr)
    qk_norm_bwd8_kernel<true><<<grid, 256, 0, s>>>(dp, sp, src.stride(0), rstd.data_ptr<float>(), w.data_ptr<float>(),
                                                   fptr(cosT), fptr(sinT), op, dsrc.stride(0), part.data_ptr<float>(),
                                                   rows, H, (int)L);
  else
    qk_norm_bwd8_kernel<false><<<grid, 256, 0, s>>>(dp, sp, src.stride(0), rstd.data_ptr<float>(), w.data_ptr<float>(),
                                                    nullptr, nullptr, op, dsrc.stride(0), part.data_ptr<float>(), rows,
                                                    H, (int)L);
  NG_LAUNCH_CHECK();
  if (dw.has_value() && dw->defined()) colsum_launch(part.data_ptr<float>(), false, grid, 64, 64, dw->data_ptr<float>(), true, s);
}

}  // namespace ng
