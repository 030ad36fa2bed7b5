// MXFP8 (OCP microscaling, e4m3 values with one E8M0 scale per 32) for the forward GEMMs of the image blocks.
//
// The reference's native-FP8 lever (baselines/PixelGen/src/models/layers/fp8_native.py:1-20, kernels K10/K11 at
// :33-78, GEMM _scaled_mm at :175-178) casts the forward GEMM inputs to e4m3 with one scale per tensor (an amax pass,
// then a cast pass) and runs cuBLASLt; the backward stays in bf16. Here the same GEMMs run on the tcgen05 block-scaled
// MMA (kind::mxf8f6f4, csrc/gemm.cu with MX tiles) with one scale per 32 values along K, so no amax pass over the whole
// tensor is needed: one pass reads bf16 and writes e4m3 values plus scales.
//
// Scale rule: e = ceil(log2(amax / 448)) over each block of 32, so amax / 2^e <= 448 (the largest finite e4m3) and no
// value saturates; the stored E8M0 byte is e + 127. An all-zero block stores 127 (scale 1).
// Scale layout (what the GEMM's TMA loads and tcgen05.cp moves to tensor memory unchanged): blocks of 128 rows x 4
// scales (512 bytes), [row blocks][K / 128][512], byte (r % 32) * 16 + (r / 32 % 4) * 4 + (k / 32 % 4). The row-block
// count is rounded up to an even number so a 256-row B tile never reads past the end; padding rows store 127.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include "common.cuh"
#include "gemm.h"
#include "status.h"

namespace ng {

// One thread per (row, 32-column block); four consecutive threads hold the four scales of one 32-bit word of the
// scale layout (K is a multiple of 128, so they sit in the same warp at lanes 4j .. 4j+3).
__global__ void mx_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int rows, int rows_pad, int K,
                                uint8_t* __restrict__ q, uint32_t* __restrict__ sf) {
  const int kb_per_row = K / 32;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool inside = t < (int64_t)rows_pad * kb_per_row;  // a lane past the end still takes part in the shuffles
  const int64_t tt = inside ? t : 0;
  const int r = (int)(tt / kb_per_row), kb = (int)(tt - (int64_t)r * kb_per_row);
  uint32_t byte = 127u;
  if (inside && r < rows) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)r * ldx + kb * 32);
    float v[32];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 u = src[j];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[8 * j + 2 * i] = bf16_bits_lo(w[i]);
        v[8 * j + 2 * i + 1] = bf16_bits_hi(w[i]);
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const int e = mx_scale_exp(amax);
    byte = (uint32_t)(e + 127);
    const float inv = ldexpf(1.f, -e);
    uint4* dst = reinterpret_cast<uint4*>(q + (int64_t)r * K + kb * 32);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint4 o;
      o.x = e4m3x4(v[16 * j + 0] * inv, v[16 * j + 1] * inv, v[16 * j + 2] * inv, v[16 * j + 3] * inv);
      o.y = e4m3x4(v[16 * j + 4] * inv, v[16 * j + 5] * inv, v[16 * j + 6] * inv, v[16 * j + 7] * inv);
      o.z = e4m3x4(v[16 * j + 8] * inv, v[16 * j + 9] * inv, v[16 * j + 10] * inv, v[16 * j + 11] * inv);
      o.w = e4m3x4(v[16 * j + 12] * inv, v[16 * j + 13] * inv, v[16 * j + 14] * inv, v[16 * j + 15] * inv);
      dst[j] = o;
    }
  }
  // gather the four scale bytes of the 32-bit word (k-blocks 4j .. 4j+3 of row r) into the lane with kb % 4 == 0
  const uint32_t b1 = __shfl_down_sync(0xffffffffu, byte, 1);
  const uint32_t b2 = __shfl_down_sync(0xffffffffu, byte, 2);
  const uint32_t b3 = __shfl_down_sync(0xffffffffu, byte, 3);
  if (inside && (kb & 3) == 0) {
    const int kt = kb >> 2, KT = K / 128;
    const int rb = r >> 7, rr = r & 127;
    const int64_t word = ((int64_t)rb * KT + kt) * 128 + (rr & 31) * 4 + (rr >> 5);
    sf[word] = byte | (b1 << 8) | (b2 << 16) | (b3 << 24);
  }
}

int64_t mx_rows_pad(int64_t rows) { return (rows + 255) / 256 * 256; }

// x [rows, K] bf16 (row stride of its own, last stride 1) -> (q [rows, K] uint8 e4m3, sf [rows_pad / 128, K / 128,
// 512] uint8)
std::vector<at::Tensor> mx_quant(const at::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "mx_quant: 2-D row-major bf16 CUDA tensor expected");
  const int64_t rows = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0, "mx_quant: K must be a multiple of 128, got ", K);
  TORCH_CHECK(x.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0,
              "mx_quant: 16-byte aligned rows expected");
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t rp = mx_rows_pad(rows);
  at::Tensor q = at::empty({rows, K}, x.options().dtype(at::kByte));
  at::Tensor sf = at::empty({rp / 128, K / 128, 512}, x.options().dtype(at::kByte));
  const int64_t threads = rp * (K / 32);
  if (threads > 0) {
    mx_quant_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), (int)rows, (int)rp, (int)K,
        q.data_ptr<uint8_t>(), reinterpret_cast<uint32_t*>(sf.data_ptr()));
    NG_LAUNCH_CHECK();
  }
  return {q, sf};
}

static const void* opt_ptr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr;
}

// out = epilogue(A_q B_q^T) with A_q [M, K], B_q [b_rows, K] e4m3 and their scale blocks (mx_quant's layout).
// epi: EPI_BF16 (out = acc + bias), EPI_GATED (out2 = y = acc + bias; out = res + gate[row / rpg] * y), EPI_SWIGLU
// (B rows [0, half_n) gate half, [half_n, 2 half_n) up half; out2 = pre, out = silu(x1) * x2; with act_q / act_sf
// given, act is also written in MXFP8, byte-identical to mx_quant(out)), EPI_SWIGLU_BWD (acc = d(act) [M, half_n],
// aux = the saved pre-activation [M, 2 half_n]; out = d(pre) [M, 2 half_n]; with act_q / act_sf given, d(pre) is also
// written in MXFP8 for the next dgrad).
void gemm_mx_torch(const at::Tensor& A, const at::Tensor& sfa, const at::Tensor& B, const at::Tensor& sfb,
                   const at::Tensor& out, int64_t epi, int64_t N, const c10::optional<at::Tensor>& out2,
                   const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& res,
                   const c10::optional<at::Tensor>& gate, int64_t rows_per_group, int64_t half_n,
                   const c10::optional<at::Tensor>& act_q, const c10::optional<at::Tensor>& act_sf,
                   const c10::optional<at::Tensor>& aux) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && out.is_cuda(), "gemm_mx: CUDA tensors expected");
  TORCH_CHECK(A.scalar_type() == at::kByte && B.scalar_type() == at::kByte && sfa.scalar_type() == at::kByte &&
                  sfb.scalar_type() == at::kByte,
              "gemm_mx: uint8 (e4m3 / e8m0) operands expected");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1) && A.stride(1) == 1 && B.stride(1) == 1,
              "gemm_mx: [M, K] and [N, K] row-major operands expected");
  const int64_t M = A.size(0), K = A.size(1);
  TORCH_CHECK(sfa.is_contiguous() && sfa.numel() >= mx_rows_pad(M) / 128 * (K / 128) * 512,
              "gemm_mx: A scale factors too small");
  TORCH_CHECK(sfb.is_contiguous() && sfb.numel() >= mx_rows_pad(B.size(0)) / 128 * (K / 128) * 512,
              "gemm_mx: B scale factors too small");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1, "gemm_mx: bf16 row-major output expected");
  if (bias.has_value() && bias->defined()) TORCH_CHECK(bias->scalar_type() == at::kFloat, "gemm_mx: fp32 bias");
  const at::cuda::CUDAGuard guard(A.device());
  GemmArgs g;
  g.mx = 1;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.A = A.data_ptr();
  g.lda = A.stride(0);
  g.B = B.data_ptr();
  g.ldb = B.stride(0);
  g.b_rows = B.size(0);
  g.sfa = sfa.data_ptr();
  g.sfb = sfb.data_ptr();
  g.epi = (int)epi;
  g.out = out.data_ptr();
  g.ldo = out.stride(0);
  if (out2.has_value() && out2->defined()) {
    g.out2 = out2->data_ptr();
    g.ldo2 = out2->stride(0);
  }
  g.bias = static_cast<const float*>(opt_ptr(bias));
  if (res.has_value() && res->defined()) {
    g.res = static_cast<const __nv_bfloat16*>(res->data_ptr());
    g.ldr = res->stride(0);
  }
  if (gate.has_value() && gate->defined()) {
    g.gate = static_cast<const __nv_bfloat16*>(gate->data_ptr());
    g.ldg = gate->stride(0);
  }
  g.rows_per_group = (int)rows_per_group;
  g.half_n = (int)half_n;
  if (aux.has_value() && aux->defined()) {
    TORCH_CHECK(epi == EPI_SWIGLU_BWD && aux->scalar_type() == at::kBFloat16 && aux->stride(1) == 1 &&
                    aux->size(0) == M && aux->size(1) == 2 * half_n,
                "gemm_mx: aux is the [M, 2 half_n] bf16 pre-activation of the SwiGLU backward");
    g.aux = static_cast<const __nv_bfloat16*>(aux->data_ptr());
    g.ld_aux = aux->stride(0);
  }
  if (act_q.has_value() && act_q->defined()) {
    TORCH_CHECK((epi == EPI_SWIGLU || epi == EPI_SWIGLU_BWD) && half_n % 128 == 0,
                "gemm_mx: the MXFP8 copy of the output is for the SwiGLU epilogues");
    const int64_t qcols = epi == EPI_SWIGLU ? half_n : 2 * half_n;
    TORCH_CHECK(act_sf.has_value() && act_sf->defined(), "gemm_mx: act scale blocks missing");
    TORCH_CHECK(act_q->scalar_type() == at::kByte && act_q->is_contiguous() && act_q->numel() == M * qcols,
                "gemm_mx: act_q must be [M, half_n] (SwiGLU) or [M, 2 half_n] (SwiGLU backward) uint8");
    TORCH_CHECK(act_sf->scalar_type() == at::kByte && act_sf->is_contiguous() &&
                    act_sf->numel() >= mx_rows_pad(M) * (qcols / 32),
                "gemm_mx: act scale blocks too small");
    g.act_q = act_q->data_ptr();
    g.act_sf = act_sf->data_ptr();
  }
  g.err = status_word();
  gemm_launch(g, at::cuda::getCurrentCUDAStream());
}

}  // namespace ng
