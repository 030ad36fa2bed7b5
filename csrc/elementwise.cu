// Memory-bound kernels around the GEMMs, for sm_100a:
//   gate_bwd      backward of out = res + gate[g] * y: dy = gate * dout, d_gate[g] = sum_rows dout * y,
//                 d_bias = sum_rows dy (deterministic chunk partials, fixed-order reduce)
//   fm_prep       flow-matching input: x_t = t x + (1 - t) eps, patchified to bf16 tokens [B*N, 3*p*p]
//   fm_loss       per-sample sum of (out - v)^2 with out = (pred - x_t)/d, v = (x - x_t)/d, d = max(1 - t, t_eps),
//                 and the gradient w.r.t. the bf16 prediction tokens in the same pass
//   patchify / unpatchify, add_rows (bf16(a + table[row % period]))
//   gather_rows   packed caption rows moved between the packed and the padded [B, Tp] layouts
// Reference: the gated residuals of JiT_T2I.py:201-210, JiTTrainer._impl_trainstep
// (baselines/PixelGen/src/diffusion/flow_matching/training_JiT.py:36-64) and patchify (JiT_T2I.py:42-52).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "finish.cuh"
#include "reduce.h"
#include "status.h"

namespace ng {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void u8(const uint4& u, float (&f)[8]) {
  f[0] = bf16_bits_lo(u.x);
  f[1] = bf16_bits_hi(u.x);
  f[2] = bf16_bits_lo(u.y);
  f[3] = bf16_bits_hi(u.y);
  f[4] = bf16_bits_lo(u.z);
  f[5] = bf16_bits_hi(u.z);
  f[6] = bf16_bits_lo(u.w);
  f[7] = bf16_bits_hi(u.w);
}
__device__ __forceinline__ uint4 p8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]);
  u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]);
  u.w = pack_bf16(f[6], f[7]);
  return u;
}

// ---------------------------------------------------------------------------------------------------- gate backward
constexpr int GB_ROWS = 32;  // rows per CTA: 1024 CTAs at 128 x 256 rows (2.3 waves of 3 CTAs per SM)

// 256 threads: RG = 256 / (C / 8) row groups (at least 1) of C / 8 threads, one 8-column vector each; a thread takes
// rows rg, rg + RG, ... of the chunk, four at a time (the loads of four rows are issued before their math), and the
// row groups' partial sums are added in shared memory in a fixed order (deterministic).
__global__ void __launch_bounds__(256) gate_bwd_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ y,
                                                       const bf16* __restrict__ gate, int64_t ldg,
                                                       bf16* __restrict__ dy, float* __restrict__ part, int M, int C,
                                                       int rpg, const int* __restrict__ cu, FinishArgs fa) {
  extern __shared__ float red[];  // [RG - 1][2][C]
  const int g = blockIdx.y, chunk = blockIdx.x;
  // rows of group g: [g rpg, (g + 1) rpg), or [cu[g], cu[g + 1]) for packed rows (a chunk past the end: zero partials)
  const int gb = cu != nullptr ? cu[g] : g * rpg;
  const int ge = cu != nullptr ? cu[g + 1] : min(g * rpg + rpg, M);
  const int r0 = gb + chunk * GB_ROWS;
  const int r1 = min(ge, r0 + GB_ROWS);
  const int nv = C >> 3;
  const int RG = max(1, (int)blockDim.x / nv);
  const int cid = g * gridDim.x + chunk;
  for (int base = 0; base < nv * RG; base += blockDim.x) {
    const int t = base + threadIdx.x;
    const int vv = t % nv, rg = t / nv;
    const bool act = t < nv * RG;
    const int c0 = vv * 8;
    float gv[8], pg[8], pb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) pg[j] = pb[j] = 0.f;
    if (act) {
      u8(*reinterpret_cast<const uint4*>(gate + (int64_t)g * ldg + c0), gv);
      for (int row = r0 + rg; row < r1; row += 4 * RG) {
        uint4 dv[4], yv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int rr = row + u * RG;
          if (rr < r1) {
            dv[u] = *reinterpret_cast<const uint4*>(dout + (int64_t)rr * C + c0);
            yv[u] = *reinterpret_cast<const uint4*>(y + (int64_t)rr * C + c0);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int rr = row + u * RG;
          if (rr < r1) {
            float d[8], yy[8], o[8], ob[8];
            u8(dv[u], d);
            u8(yv[u], yy);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              pg[j] += d[j] * yy[j];
              o[j] = gv[j] * d[j];
            }
            const uint4 packed = p8(o);
            *reinterpret_cast<uint4*>(dy + (int64_t)rr * C + c0) = packed;
            u8(packed, ob);  // the bias sees the rounded dy that the GEMMs consume
#pragma unroll
            for (int j = 0; j < 8; ++j) pb[j] += ob[j];
          }
        }
      }
    }
    // row groups 1.. hand their sums to group 0 (a block whose vectors wrap, RG == 1, skips this)
    if (RG > 1) {
      if (act && rg > 0) {
        float* dst = red + (int64_t)(rg - 1) * 2 * C;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          dst[c0 + j] = pg[j];
          dst[C + c0 + j] = pb[j];
        }
      }
      __syncthreads();
      if (act && rg == 0) {
        for (int k = 1; k < RG; ++k) {
          const float* src = red + (int64_t)(k - 1) * 2 * C;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            pg[j] += src[c0 + j];
            pb[j] += src[C + c0 + j];
          }
        }
      }
      __syncthreads();
    }
    if (act && rg == 0) {
      float* pp = part + (int64_t)cid * 2 * C;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        pp[c0 + j] = pg[j];
        pp[C + c0 + j] = pb[j];
      }
    }
  }
  // the group's last CTA writes d_gate[g] and the group's d_bias row: fixed order, no group-sum launch
  finish_partials<2>(part, 2 * C, C, gridDim.x, g, fa);
}

// ---------------------------------------------------------------------------------------------- image input
// uint8 HWC images [B, H, W, 3] -> fp32 CHW in [-1, 1] with the reference's formula (ToTensor, then Normalize(0.5,
// 0.5): (u / 255 - 0.5) / 0.5), rounded as PyTorch evaluates it on the device: a division by a scalar is a
// multiplication by the scalar's fp32 reciprocal, each operation rounded on its own (no fused multiply-add), and the
// division by 0.5 is the exact multiplication by 2. A thread per 8 pixels of a row: three 8-byte loads, two 16-byte
// stores per channel. W % 8 == 0.
__global__ void u8_to_unit_kernel(const uint8_t* __restrict__ img, float* __restrict__ out, int64_t rows, int H,
                                  int W) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int w8 = W / 8;
  if (i >= rows * w8) return;
  const int64_t bh = i / w8;
  const int x0 = (int)(i - bh * w8) * 8;
  const int64_t b = bh / H;
  const int h = (int)(bh - b * H);
  const uint2* src = reinterpret_cast<const uint2*>(img + (bh * W + x0) * 3);
  uint8_t px[24];
#pragma unroll
  for (int k = 0; k < 3; ++k) *reinterpret_cast<uint2*>(px + 8 * k) = src[k];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __fsub_rn(__fmul_rn((float)px[3 * j + c], 1.0f / 255.0f), 0.5f) * 2.0f;
    float4* dst = reinterpret_cast<float4*>(out + ((b * 3 + c) * H + h) * (int64_t)W + x0);
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

void u8_to_unit(const at::Tensor& img, const at::Tensor& out) {
  TORCH_CHECK(img.is_cuda() && img.scalar_type() == at::kByte && img.is_contiguous() && img.dim() == 4 &&
                  img.size(3) == 3 && img.size(2) % 8 == 0,
              "u8_to_unit: contiguous uint8 [B, H, W, 3] with W % 8 == 0");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.size(0) == img.size(0) &&
                  out.size(1) == 3 && out.size(2) == img.size(1) && out.size(3) == img.size(2),
              "u8_to_unit: fp32 [B, 3, H, W] output");
  const at::cuda::CUDAGuard guard(img.device());
  const int64_t rows = img.size(0) * img.size(1);
  const int H = img.size(1), W = img.size(2);
  const int64_t n = rows * (W / 8);
  if (n == 0) return;
  u8_to_unit_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      img.data_ptr<uint8_t>(), out.data_ptr<float>(), rows, H, W);
  NG_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------------------------- flow matching
// token n of sample b, element e = c*p*p + py*p + px  <->  pixel (b, c, (n / gw)*p + py, (n % gw)*p + px)
// each thread handles 8 consecutive elements (same c, py; px in [8k, 8k+8)): needs p % 8 == 0
__global__ void fm_prep_kernel(const float* __restrict__ x, const float* __restrict__ noise,
                               const float* __restrict__ t, bf16* __restrict__ xt_tok, int B, int Cin, int H, int W,
                               int p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // index of an 8-element group
  const int D = Cin * p * p, gw = W / p, N = (H / p) * gw;
  const int64_t total = (int64_t)B * N * D / 8;
  if (i >= total) return;
  const int64_t e0 = i * 8;
  const int64_t tok = e0 / D;
  const int e = (int)(e0 - tok * D);
  const int b = (int)(tok / N), n = (int)(tok - (int64_t)b * N);
  const int c = e / (p * p), py = (e / p) % p, px = e % p;
  const int yy = (n / gw) * p + py, xx = (n % gw) * p + px;
  const int64_t pix = (((int64_t)b * Cin + c) * H + yy) * W + xx;
  const float tb = t[b];
  const float4 xa = *reinterpret_cast<const float4*>(x + pix), xb = *reinterpret_cast<const float4*>(x + pix + 4);
  const float4 na = *reinterpret_cast<const float4*>(noise + pix), nb = *reinterpret_cast<const float4*>(noise + pix + 4);
  const float s = 1.f - tb;
  float o[8] = {tb * xa.x + na.x * s, tb * xa.y + na.y * s, tb * xa.z + na.z * s, tb * xa.w + na.w * s,
                tb * xb.x + nb.x * s, tb * xb.y + nb.y * s, tb * xb.z + nb.z * s, tb * xb.w + nb.w * s};
  *reinterpret_cast<uint4*>(xt_tok + e0) = p8(o);
}

// per-(sample, block) partial sums; grid.x = blocks per sample, grid.y = B
__global__ void __launch_bounds__(256) fm_loss_kernel(const bf16* __restrict__ pred, const float* __restrict__ x,
                                                      const float* __restrict__ noise, const float* __restrict__ t,
                                                      bf16* __restrict__ dpred, float* __restrict__ part, int Cin,
                                                      int H, int W, int p, float t_eps, float grad_scale) {
  __shared__ float red[8];
  const int b = blockIdx.y;
  const int D = Cin * p * p, gw = W / p, N = (H / p) * gw;
  const int64_t per_sample = (int64_t)N * D / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float acc = 0.f;
  if (i < per_sample) {
    const int64_t e0 = i * 8;
    const int n = (int)(e0 / D);
    const int e = (int)(e0 - (int64_t)n * D);
    const int c = e / (p * p), py = (e / p) % p, px = e % p;
    const int yy = (n / gw) * p + py, xx = (n % gw) * p + px;
    const int64_t pix = (((int64_t)b * Cin + c) * H + yy) * W + xx;
    const float tb = t[b];
    const float den = fmaxf(1.f - tb, t_eps);
    float xv[8], nv[8], pv[8], g[8];
    *reinterpret_cast<float4*>(xv) = *reinterpret_cast<const float4*>(x + pix);
    *reinterpret_cast<float4*>(xv + 4) = *reinterpret_cast<const float4*>(x + pix + 4);
    *reinterpret_cast<float4*>(nv) = *reinterpret_cast<const float4*>(noise + pix);
    *reinterpret_cast<float4*>(nv + 4) = *reinterpret_cast<const float4*>(noise + pix + 4);
    const int64_t tokoff = ((int64_t)b * N + n) * D + e;
    u8(*reinterpret_cast<const uint4*>(pred + tokoff), pv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float xt = tb * xv[j] + nv[j] * (1.f - tb);
      const float out = (pv[j] - xt) / den;
      const float v = (xv[j] - xt) / den;
      const float d = out - v;
      acc += d * d;
      g[j] = grad_scale * 2.f * d / den;
    }
    if (dpred != nullptr) *reinterpret_cast<uint4*>(dpred + tokoff) = p8(g);
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int k = 0; k < 8; ++k) s += red[k];
    part[(int64_t)b * gridDim.x + blockIdx.x] = s;
  }
}

__global__ void fm_loss_reduce(const float* __restrict__ part, int nblk, float* __restrict__ per_sample, float inv_d) {
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int k = 0; k < nblk; ++k) s += part[(int64_t)b * nblk + k];
    per_sample[b] = s * inv_d;
  }
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(bf16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

// tokens [B*N, Cin*p*p] (bf16) <-> image [B, Cin, H, W] (fp32 or bf16 out)
template <typename Tin, typename Tout, bool TO_TOKENS>
__global__ void patch_kernel(const Tin* __restrict__ src, Tout* __restrict__ dst, int B, int Cin, int H, int W, int p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int D = Cin * p * p, gw = W / p, N = (H / p) * gw;
  const int64_t total = (int64_t)B * N * D;
  if (i >= total) return;
  const int64_t tok = i / D;
  const int e = (int)(i - tok * D);
  const int b = (int)(tok / N), n = (int)(tok - (int64_t)b * N);
  const int c = e / (p * p), py = (e / p) % p, px = e % p;
  const int64_t pix = (((int64_t)b * Cin + c) * H + (n / gw) * p + py) * W + (n % gw) * p + px;
  if (TO_TOKENS)
    dst[i] = from_f<Tout>(to_f(src[pix]));
  else
    dst[pix] = from_f<Tout>(to_f(src[i]));
}

// out[row] = bf16(a[row] + table[row % period]) (fp32 or bf16 table [period, C])
template <typename TT>
__global__ void add_rows_kernel(const bf16* __restrict__ a, const TT* __restrict__ table, bf16* __restrict__ out,
                                int64_t rows, int C, int period) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int nv = C / 8;
  if (i >= rows * nv) return;
  const int64_t row = i / nv;
  const int c0 = (int)(i - row * nv) * 8;
  float f[8];
  u8(*reinterpret_cast<const uint4*>(a + row * C + c0), f);
  const TT* tr = table + (int64_t)(row % period) * C + c0;
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] += to_f(tr[j]);
  *reinterpret_cast<uint4*>(out + row * C + c0) = p8(f);
}

// ====================================================================================================== torch glue
void gate_bwd(const at::Tensor& dout, const at::Tensor& y, const at::Tensor& gate, const at::Tensor& dy,
              const c10::optional<at::Tensor>& dgate, const c10::optional<at::Tensor>& dbias, int64_t rpg,
              const c10::optional<at::Tensor>& cu, int64_t max_rows) {
  TORCH_CHECK(dout.is_contiguous() && y.is_contiguous() && dy.is_contiguous() && gate.stride(1) == 1,
              "gate_bwd: layouts");
  const at::cuda::CUDAGuard guard(dout.device());
  const int M = dout.size(0), C = dout.size(1);
  TORCH_CHECK(C % 8 == 0, "gate_bwd: C % 8");
  const bool packed = cu.has_value() && cu->defined();
  const int* cup = nullptr;
  if (packed) {
    TORCH_CHECK(cu->scalar_type() == at::kInt && cu->is_contiguous() && cu->numel() >= 2 && cu->is_cuda() &&
                    max_rows > 0,
                "gate_bwd: cu must be a [G + 1] int32 CUDA tensor of row offsets, with max_rows > 0");
    cup = cu->data_ptr<int>();
  }
  const int G = packed ? (int)cu->numel() - 1 : (M + (int)rpg - 1) / (int)rpg;
  TORCH_CHECK(G <= 65535, "gate_bwd: at most 65535 groups");
  const int chunks = ((packed ? (int)max_rows : (int)rpg) + GB_ROWS - 1) / GB_ROWS;
  auto s = at::cuda::getCurrentCUDAStream();
  // chunk partials, then the group rows of the d_bias sums
  at::Tensor part = at::empty({(int64_t)G * chunks * 2 * C + (int64_t)G * C}, dout.options().dtype(at::kFloat));
  const int RG = std::max(1, 256 / (C / 8));
  const size_t smem = RG > 1 ? (size_t)(RG - 1) * 2 * C * sizeof(float) : 0;
  FinishArgs fa{};
  fa.gout[0] = (dgate.has_value() && dgate->defined()) ? dgate->data_ptr<float>() : nullptr;
  fa.gld[0] = fa.gout[0] != nullptr ? dgate->stride(0) : 0;
  fa.scratch = part.data_ptr<float>() + (int64_t)G * chunks * 2 * C;
  const bool in_kernel = chunks <= kFinishMaxChunks;  // as in rms_mod_bwd: no long serial tail
  fa.cnt = in_kernel ? finish_counters(s, G) : nullptr;
  gate_bwd_kernel<<<dim3(chunks, G), 256, smem, s>>>(
      reinterpret_cast<const bf16*>(dout.data_ptr()), reinterpret_cast<const bf16*>(y.data_ptr()),
      reinterpret_cast<const bf16*>(gate.data_ptr()), gate.stride(0), reinterpret_cast<bf16*>(dy.data_ptr()),
      part.data_ptr<float>(), M, C, (int)rpg, cup, fa);
  NG_LAUNCH_CHECK();
  float* db = (dbias.has_value() && dbias->defined()) ? dbias->data_ptr<float>() : nullptr;
  if (in_kernel) {  // d_bias: the column sums of the G group rows the kernel left in the scratch
    if (db != nullptr) colsum_launch(fa.scratch, false, G, C, C, db, true, s);
    return;
  }
  const float* pp = part.data_ptr<float>();
  group_sum_launch(pp, G, chunks, C, 2 * C, fa.gout[0], fa.gld[0], s);
  if (db != nullptr) colsum_launch(pp + C, false, (int64_t)G * chunks, C, 2 * C, db, true, s);
}

void fm_prep(const at::Tensor& x, const at::Tensor& noise, const at::Tensor& t, const at::Tensor& xt_tok, int64_t p) {
  TORCH_CHECK(x.is_contiguous() && noise.is_contiguous() && x.scalar_type() == at::kFloat, "fm_prep: fp32 images");
  TORCH_CHECK(p % 8 == 0, "fm_prep: patch size must be a multiple of 8");
  const at::cuda::CUDAGuard guard(x.device());
  const int B = x.size(0), Cin = x.size(1), H = x.size(2), W = x.size(3);
  const int64_t groups = x.numel() / 8;
  fm_prep_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), noise.data_ptr<float>(), t.data_ptr<float>(), reinterpret_cast<bf16*>(xt_tok.data_ptr()),
      B, Cin, H, W, (int)p);
  NG_LAUNCH_CHECK();
}

void fm_loss(const at::Tensor& pred, const at::Tensor& x, const at::Tensor& noise, const at::Tensor& t,
             const c10::optional<at::Tensor>& dpred, const at::Tensor& per_sample, int64_t p, double t_eps,
             double grad_scale) {
  const at::cuda::CUDAGuard guard(x.device());
  const int B = x.size(0), Cin = x.size(1), H = x.size(2), W = x.size(3);
  const int64_t per = x.numel() / B / 8;
  const int nblk = (int)((per + 255) / 256);
  auto s = at::cuda::getCurrentCUDAStream();
  at::Tensor part = at::empty({(int64_t)B * nblk}, x.options());
  bf16* dp = (dpred.has_value() && dpred->defined()) ? reinterpret_cast<bf16*>(dpred->data_ptr()) : nullptr;
  fm_loss_kernel<<<dim3(nblk, B), 256, 0, s>>>(reinterpret_cast<const bf16*>(pred.data_ptr()), x.data_ptr<float>(),
                                               noise.data_ptr<float>(), t.data_ptr<float>(), dp,
                                               part.data_ptr<float>(), Cin, H, W, (int)p, (float)t_eps,
                                               (float)grad_scale);
  NG_LAUNCH_CHECK();
  fm_loss_reduce<<<B, 32, 0, s>>>(part.data_ptr<float>(), nblk, per_sample.data_ptr<float>(),
                                  1.f / (float)(x.numel() / B));
  NG_LAUNCH_CHECK();
}

void patchify(const at::Tensor& img, const at::Tensor& tok, int64_t p) {
  const at::cuda::CUDAGuard guard(img.device());
  const int B = img.size(0), Cin = img.size(1), H = img.size(2), W = img.size(3);
  const int64_t n = img.numel();
  auto s = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(tok.scalar_type() == at::kBFloat16, "patchify: bf16 tokens");
  if (img.scalar_type() == at::kFloat)
    patch_kernel<float, bf16, true><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        img.data_ptr<float>(), reinterpret_cast<bf16*>(tok.data_ptr()), B, Cin, H, W, (int)p);
  else
    patch_kernel<bf16, bf16, true><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<const bf16*>(img.data_ptr()), reinterpret_cast<bf16*>(tok.data_ptr()), B, Cin, H, W, (int)p);
  NG_LAUNCH_CHECK();
}

void unpatchify(const at::Tensor& tok, const at::Tensor& img, int64_t p) {
  const at::cuda::CUDAGuard guard(img.device());
  const int B = img.size(0), Cin = img.size(1), H = img.size(2), W = img.size(3);
  const int64_t n = img.numel();
  auto s = at::cuda::getCurrentCUDAStream();
  if (img.scalar_type() == at::kFloat)
    patch_kernel<bf16, float, false><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<const bf16*>(tok.data_ptr()), img.data_ptr<float>(), B, Cin, H, W, (int)p);
  else
    patch_kernel<bf16, bf16, false><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<const bf16*>(tok.data_ptr()), reinterpret_cast<bf16*>(img.data_ptr()), B, Cin, H, W, (int)p);
  NG_LAUNCH_CHECK();
}

void add_rows(const at::Tensor& a, const at::Tensor& table, const at::Tensor& out, int64_t period) {
  TORCH_CHECK(a.is_contiguous() && table.is_contiguous() && out.is_contiguous(), "add_rows: contiguous");
  const at::cuda::CUDAGuard guard(a.device());
  const int64_t rows = a.size(0);
  const int C = a.size(1);
  TORCH_CHECK(C % 8 == 0, "add_rows: C % 8");
  const int64_t n = rows * (C / 8);
  auto s = at::cuda::getCurrentCUDAStream();
  if (table.scalar_type() == at::kFloat)
    add_rows_kernel<float><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<const bf16*>(a.data_ptr()), table.data_ptr<float>(), reinterpret_cast<bf16*>(out.data_ptr()),
        rows, C, (int)period);
  else
    add_rows_kernel<bf16><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<const bf16*>(a.data_ptr()), reinterpret_cast<const bf16*>(table.data_ptr()),
        reinterpret_cast<bf16*>(out.data_ptr()), rows, C, (int)period);
  NG_LAUNCH_CHECK();
}

// --------------------------------------------------------------------------------------------- packed caption rows
// gather_rows: out[r] = src[idx[r]] for bf16 rows of C values (16-byte vectors), zeros where idx[r] < 0. Moves packed
// caption rows into the padded [B, Tp] layout the attention reads and back (JiT_T2I.py:54-65 of the reference).
__global__ void gather_rows_kernel(const bf16* __restrict__ src, int64_t lds, const int* __restrict__ idx,
                                   bf16* __restrict__ out, int64_t ldo, int64_t rows, int nv) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * nv) return;
  const int64_t r = i / nv;
  const int v = (int)(i - r * nv);
  const int s = idx[r];
  uint4 val = make_uint4(0u, 0u, 0u, 0u);
  if (s >= 0) val = reinterpret_cast<const uint4*>(src + (int64_t)s * lds)[v];
  reinterpret_cast<uint4*>(out + r * ldo)[v] = val;
}

void gather_rows(const at::Tensor& src, const at::Tensor& idx, const at::Tensor& out) {
  TORCH_CHECK(src.dim() == 2 && out.dim() == 2 && src.size(1) == out.size(1) && src.stride(1) == 1 &&
                  out.stride(1) == 1 && src.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
              "gather_rows: 2-D bf16 rows with unit column stride");
  TORCH_CHECK(idx.scalar_type() == at::kInt && idx.is_contiguous() && idx.numel() == out.size(0),
              "gather_rows: idx [rows of out] int32");
  const int C = src.size(1);
  TORCH_CHECK(C % 8 == 0 && src.stride(0) % 8 == 0 && out.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "gather_rows: 16-byte aligned rows");
  const at::cuda::CUDAGuard guard(src.device());
  const int64_t rows = out.size(0);
  const int nv = C / 8;
  const int64_t n = rows * nv;
  if (n == 0) return;
  gather_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(src.data_ptr()), src.stride(0), idx.data_ptr<int>(),
      reinterpret_cast<bf16*>(out.data_ptr()), out.stride(0), rows, nv);
  NG_LAUNCH_CHECK();
}

}  // namespace ng
