"""MXFP8 (e4m3 values, one E8M0 scale per 32 along K) operands and the block-scaled GEMMs of the image blocks.

Role of the reference's native-FP8 lever (baselines/PixelGen/src/models/layers/fp8_native.py:1-20; casts K10/K11 at
:33-78, GEMM :175-178, module swap `convert_native` :290-318): the forward GEMMs of the image blocks (qkv_x, proj, w12,
w3) read e4m3 inputs, the backward stays in bf16 (dgrad from the bf16 weight, wgrad from the bf16 activations). Here
the scales are per 32 values (OCP MX) instead of per tensor, the GEMM is the tcgen05 block-scaled MMA
(csrc/gemm.cu, MX tiles) with the same fused epilogues as the bf16 path, and the cast is one pass (csrc/mx.cu).

CPU tensors take a PyTorch restatement of the same quantization (bit-identical values and scales) and dequantize for
the GEMMs, which is what the CPU tests and oracles use.
"""
import torch

from .._ext import ext
from . import gemm as G

E4M3_MAX = 448.0


def rows_pad(rows):
    return (rows + 255) // 256 * 256


class MX:
    """An MXFP8 matrix: q [rows, K] uint8 (e4m3 bits), sf [rows_pad / 128, K / 128, 512] uint8 (E8M0 bytes in the
    GEMM's 128-row x 4-scale blocks, byte (r % 32) * 16 + (r / 32 % 4) * 4 + (k / 32 % 4))."""

    __slots__ = ("q", "sf")

    def __init__(self, q, sf):
        self.q, self.sf = q, sf

    @property
    def shape(self):
        return self.q.shape

    def scales(self):
        """Scale exponents as a [rows, K / 32] int tensor (E8M0 byte - 127)."""
        R, K = self.q.shape
        s = self.sf.view(-1, K // 128, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(-1, K // 32)
        return s[:R].long() - 127

    def dequant(self):
        """fp32 values q * 2^e."""
        R, K = self.q.shape
        v = self.q.view(torch.float8_e4m3fn).float().view(R, K // 32, 32)
        return (v * torch.pow(2.0, self.scales().float()).unsqueeze(-1)).view(R, K)


def _quant_torch(x):
    R, K = x.shape
    xb = x.float().reshape(R, K // 32, 32)
    amax = xb.abs().amax(-1)
    m, E = torch.frexp(amax / E4M3_MAX)  # amax / 448 = m 2^E, m in [0.5, 1): ceil(log2) = E - (m == 0.5)
    e = torch.where(m == 0.5, E - 1, E)
    e = torch.where(amax > 0, e, torch.zeros_like(e)).clamp(-127, 127)
    v = (xb * torch.pow(2.0, -e.float()).unsqueeze(-1)).clamp(-E4M3_MAX, E4M3_MAX)
    q = v.to(torch.float8_e4m3fn).view(torch.uint8).reshape(R, K)
    Rp = rows_pad(R)
    s = torch.full((Rp, K // 32), 127, dtype=torch.uint8, device=x.device)
    s[:R] = (e + 127).to(torch.uint8)
    sf = s.view(Rp // 128, 4, 32, K // 128, 4).permute(0, 3, 2, 1, 4).reshape(Rp // 128, K // 128, 512)
    return MX(q, sf.contiguous())


def quant(x):
    """bf16 [rows, K] (K a multiple of 128, row-major) -> MX."""
    assert x.dim() == 2 and x.shape[1] % 128 == 0, "MX quantization needs K % 128 == 0"
    if not x.is_cuda:
        return _quant_torch(x)
    q, sf = ext().mx_quant(x)
    return MX(q, sf)


# ------------------------------------------------------------------------------------------------------- GEMMs
def linear(xq, wq, bias=None):
    """bf16(dequant(xq) @ dequant(wq)^T + bias) -> [M, N]."""
    if not xq.q.is_cuda:
        return G.linear(xq.dequant(), wq.dequant(), bias)
    M, N = xq.shape[0], wq.shape[0]
    out = torch.empty(M, N, device=xq.q.device, dtype=torch.bfloat16)
    ext().gemm_mx(xq.q, xq.sf, wq.q, wq.sf, out, G.EPI_BF16, N, None, bias, None, None, 1, 0, None, None, None)
    return out


def linear_gated_residual(xq, wq, bias, res, gate, rows_per_group):
    """y = bf16(x W^T + bias); out = bf16(res + gate[row // rows_per_group] * y). Returns (out, y)."""
    if not xq.q.is_cuda:
        return G.linear_gated_residual(xq.dequant(), wq.dequant(), bias, res, gate, rows_per_group)
    M, N = xq.shape[0], wq.shape[0]
    out = torch.empty(M, N, device=xq.q.device, dtype=torch.bfloat16)
    y = torch.empty(M, N, device=xq.q.device, dtype=torch.bfloat16)
    ext().gemm_mx(xq.q, xq.sf, wq.q, wq.sf, out, G.EPI_GATED, N, y, bias, res, gate, rows_per_group, 0, None, None,
                  None)
    return out, y


def empty_like_rows(rows, K, device):
    """An MX buffer for a [rows, K] matrix written by a kernel: scale rows past `rows` (padding) hold scale 1."""
    rp = rows_pad(rows)
    q = torch.empty(rows, K, device=device, dtype=torch.uint8)
    shape = (rp // 128, K // 128, 512)
    sf = (torch.empty(shape, device=device, dtype=torch.uint8) if rp == rows
          else torch.full(shape, 127, device=device, dtype=torch.uint8))
    return MX(q, sf)


def swiglu_linear(xq, w12q, quant_act=False):
    """pre = bf16(x W12^T) [M, 2H]; act = bf16(silu(pre[:, :H]) * pre[:, H:]). Returns (act, pre), or with quant_act
    (act, pre, actq): actq is act in MXFP8, written by the GEMM's epilogue (equal to quant(act))."""
    if not xq.q.is_cuda:
        act, pre = G.swiglu_linear(xq.dequant(), w12q.dequant())
        return (act, pre, quant(act)) if quant_act else (act, pre)
    M, H2 = xq.shape[0], w12q.shape[0]
    H = H2 // 2
    act = torch.empty(M, H, device=xq.q.device, dtype=torch.bfloat16)
    pre = torch.empty(M, H2, device=xq.q.device, dtype=torch.bfloat16)
    aq = empty_like_rows(M, H, xq.q.device) if quant_act else None
    ext().gemm_mx(xq.q, xq.sf, w12q.q, w12q.sf, act, G.EPI_SWIGLU, H2, pre, None, None, None, 1, H,
                  aq.q if aq is not None else None, aq.sf if aq is not None else None, None)
    return (act, pre, aq) if quant_act else (act, pre)


def swiglu_dgrad(dyq, w3tq, pre, quant_out=False):
    """Backward of act = silu(pre[:, :H]) * pre[:, H:] through y = act W3^T, in MXFP8 (the reference's phase-2 FP8
    MLP backward, fp8_native.py:236-266): d(act) = dy W3 from dy's MX copy and W3^T's ([H, C]), and the SwiGLU
    backward in the GEMM's epilogue. Returns d(pre) [M, 2H] bf16, or with quant_out (dpre, dpre's MX copy written by
    the same epilogue, equal to quant(dpre))."""
    if not dyq.q.is_cuda:
        dpre = G.swiglu_dgrad(dyq.dequant().to(torch.bfloat16), w3tq.dequant().t().contiguous().to(torch.bfloat16),
                              pre)
        return (dpre, quant(dpre)) if quant_out else dpre
    M, H = dyq.shape[0], w3tq.shape[0]
    dpre = torch.empty(M, 2 * H, device=dyq.q.device, dtype=torch.bfloat16)
    dq = empty_like_rows(M, 2 * H, dyq.q.device) if quant_out else None
    ext().gemm_mx(dyq.q, dyq.sf, w3tq.q, w3tq.sf, dpre, G.EPI_SWIGLU_BWD, H, None, None, None, None, 1, H,
                  dq.q if dq is not None else None, dq.sf if dq is not None else None, pre)
    return (dpre, dq) if quant_out else dpre
