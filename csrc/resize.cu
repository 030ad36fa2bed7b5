// Pillow's 8-bit separable bicubic passes for a batch of crops (the GPU half of nano_gpic_b200/data/pil_resize.py).
//
// Role of the reference's lever C kernels (baselines/PixelGen/src/data/dataset/pil_exact_gpu.py:17-122): every
// output value of a pass is clip8((2^21 + sum_j in[xmin + j] * kk[j]) >> 22) with an int32 sum, the arithmetic of
// Pillow's Resample.c, so the result equals Pillow's byte for byte whenever the tables (built on the host) do.
// One thread per output pixel (3 channels); each sample has its own source size and tables, described by a row of
// `desc` (int64 x 16): [src_off, h, w, axis0, ksize0, tab0_off, tmp_off, mid_h, mid_w, axis1, ksize1, tab1_off].
// A pass's table is xmin[size], xlen[size], kk[size * ksize] (int32). Pass 0 reads the source and writes the
// intermediate; pass 1 reads the intermediate and writes out[b] (size x size x 3).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "status.h"

namespace ng {

__global__ void resize_pass_kernel(const uint8_t* __restrict__ src_all, const uint8_t* __restrict__ tmp_all,
                                   const int32_t* __restrict__ tab_all, const int64_t* __restrict__ desc,
                                   uint8_t* __restrict__ tmp_out, uint8_t* __restrict__ out, int size, int pass) {
  const int b = blockIdx.y;
  const int64_t* d = desc + (int64_t)b * 16;
  const int ih = pass == 0 ? (int)d[1] : (int)d[7];  // input rows / columns of this pass
  const int iw = pass == 0 ? (int)d[2] : (int)d[8];
  const int axis = pass == 0 ? (int)d[3] : (int)d[9];
  const int ksize = pass == 0 ? (int)d[4] : (int)d[10];
  const int32_t* tab = tab_all + (pass == 0 ? d[5] : d[11]);
  const uint8_t* in = pass == 0 ? src_all + d[0] : tmp_all + d[6];
  uint8_t* dst = pass == 0 ? tmp_out + d[6] : out + (int64_t)b * size * size * 3;
  // output shape: the pass replaces the extent along its axis by `size`
  const int oh = axis == 0 ? size : ih, ow = axis == 0 ? iw : size;
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= (int64_t)oh * ow) return;
  const int oy = (int)(p / ow), ox = (int)(p - (int64_t)oy * ow);
  const int o = axis == 0 ? oy : ox;  // output index along the pass axis
  const int xmin = tab[o], xlen = tab[size + o];
  const int32_t* kk = tab + 2 * size + (int64_t)o * ksize;
  int32_t s0 = 1 << 21, s1 = 1 << 21, s2 = 1 << 21;
  for (int j = 0; j < xlen; ++j) {
    const int64_t q = axis == 0 ? ((int64_t)(xmin + j) * iw + ox) * 3 : ((int64_t)oy * iw + xmin + j) * 3;
    const int32_t w = kk[j];
    s0 += (int32_t)in[q] * w;
    s1 += (int32_t)in[q + 1] * w;
    s2 += (int32_t)in[q + 2] * w;
  }
  uint8_t* r = dst + p * 3;
  r[0] = (uint8_t)min(255, max(0, s0 >> 22));
  r[1] = (uint8_t)min(255, max(0, s1 >> 22));
  r[2] = (uint8_t)min(255, max(0, s2 >> 22));
}

void resize_passes(const at::Tensor& src, const at::Tensor& tab, const at::Tensor& desc, const at::Tensor& tmp,
                   const at::Tensor& out, int64_t max_h, int64_t max_w) {
  TORCH_CHECK(src.is_cuda() && tab.is_cuda() && desc.is_cuda() && tmp.is_cuda() && out.is_cuda(),
              "resize_passes: CUDA tensors expected");
  TORCH_CHECK(src.scalar_type() == at::kByte && tab.scalar_type() == at::kInt && desc.scalar_type() == at::kLong &&
                  out.scalar_type() == at::kByte && out.dim() == 4 && out.size(3) == 3 && out.size(1) == out.size(2),
              "resize_passes: uint8 sources, int32 tables, int64 descriptors, [B, S, S, 3] uint8 output");
  TORCH_CHECK(desc.dim() == 2 && desc.size(1) == 16 && desc.size(0) == out.size(0), "resize_passes: [B, 16] desc");
  const at::cuda::CUDAGuard guard(src.device());
  const int B = (int)out.size(0), S = (int)out.size(1);
  if (B == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int64_t px0 = (int64_t)S * std::max(max_h, max_w);  // bound of the first pass's output pixels
  const int64_t px1 = (int64_t)S * S;
  resize_pass_kernel<<<dim3((unsigned)((px0 + 255) / 256), B), 256, 0, stream>>>(
      src.data_ptr<uint8_t>(), tmp.data_ptr<uint8_t>(), tab.data_ptr<int32_t>(), desc.data_ptr<int64_t>(),
      tmp.data_ptr<uint8_t>(), out.data_ptr<uint8_t>(), S, 0);
  NG_LAUNCH_CHECK();
  resize_pass_kernel<<<dim3((unsigned)((px1 + 255) / 256), B), 256, 0, stream>>>(
      src.data_ptr<uint8_t>(), tmp.data_ptr<uint8_t>(), tab.data_ptr<int32_t>(), desc.data_ptr<int64_t>(),
      tmp.data_ptr<uint8_t>(), out.data_ptr<uint8_t>(), S, 1);
  NG_LAUNCH_CHECK();
}

}  // namespace ng
