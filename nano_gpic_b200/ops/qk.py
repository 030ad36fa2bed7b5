"""Per-head RMSNorm of queries/keys with the 2D RoPE applied in the same pass (forward and backward).

For one head vector x (64 values) at image position p:
    xn = w * x * rstd,  rstd = 1 / sqrt(mean(x^2) + eps)
    out[2j]   = xn[2j] cos(p, j) - xn[2j+1] sin(p, j)
    out[2j+1] = xn[2j] sin(p, j) + xn[2j+1] cos(p, j)          (no rotation when the tables are None)
cos/sin are the real and imaginary parts of the reference's precompute_freqs_cis_ex2d table, [L, 32].

Reference sites: q_norm/k_norm + apply_rotary_emb_real in Attention.forward (baselines/PixelGen/src/models/transformer/
JiT_T2I.py:141-166, baselines/PixelGen/src/models/layers/rope.py:53-69) and the Triton fused QK prep of lever K2
(baselines/PixelGen/src/models/layers/fused_qk.py:55-200).
"""
import torch

from .._ext import ext

HEAD = 64


def _rope_cpu(xn, cos, sin, L):
    rows = xn.shape[0]
    H = xn.shape[1] // HEAD
    pos = torch.arange(rows) % L
    c, s = cos[pos][:, None, :].float(), sin[pos][:, None, :].float()
    v = xn.view(rows, H, HEAD // 2, 2)
    a, b = v[..., 0], v[..., 1]
    return torch.stack([a * c - b * s, a * s + b * c], -1).reshape(rows, H * HEAD)


def _irope_cpu(d, cos, sin, L):
    rows = d.shape[0]
    H = d.shape[1] // HEAD
    pos = torch.arange(rows) % L
    c, s = cos[pos][:, None, :].float(), sin[pos][:, None, :].float()
    v = d.view(rows, H, HEAD // 2, 2)
    a, b = v[..., 0], v[..., 1]
    return torch.stack([a * c + b * s, -a * s + b * c], -1).reshape(rows, H * HEAD)


def qk_norm_fwd(src, w, cos=None, sin=None, L=1, eps=1e-6):
    """src [rows, H*64] bf16 view (row stride free, last stride 1). Returns (out [rows, H*64] bf16 contiguous,
    rstd [rows, H] fp32)."""
    rows, C = src.shape
    H = C // HEAD
    if not src.is_cuda:
        x = src.float().view(rows, H, HEAD)
        rstd = torch.rsqrt(x.pow(2).mean(-1) + eps)
        xn = (w.float() * x * rstd[..., None]).reshape(rows, C)
        if cos is not None:
            xn = _rope_cpu(xn, cos, sin, L)
        return xn.to(torch.bfloat16), rstd
    out = torch.empty(rows, C, device=src.device, dtype=torch.bfloat16)
    rstd = torch.empty(rows, H, device=src.device, dtype=torch.float32)
    ext().qk_norm_fwd(src, w, cos, sin, out, rstd, L, eps)
    return out, rstd


def qk_norm_bwd(dout, src, rstd, w, cos=None, sin=None, L=1, dsrc=None, dw_acc=None):
    """Backward of qk_norm_fwd. dsrc: [rows, H*64] bf16 view to write (a slice of the fused projection's gradient);
    dw_acc [64] fp32 accumulates the weight gradient (summed over rows and heads)."""
    rows, C = src.shape
    H = C // HEAD
    if not src.is_cuda:
        d = dout.float()
        if cos is not None:
            d = _irope_cpu(d, cos, sin, L)
        d = d.view(rows, H, HEAD)
        xh = src.float().view(rows, H, HEAD) * rstd[..., None]
        if dw_acc is not None:
            dw_acc.add_((d * xh).sum((0, 1)))
        dxh = d * w.float()
        dx = rstd[..., None] * (dxh - xh * (dxh * xh).mean(-1, keepdim=True))
        dx = dx.reshape(rows, C).to(torch.bfloat16)
        if dsrc is None:
            return dx
        dsrc.copy_(dx)
        return dsrc
    if dsrc is None:
        dsrc = torch.empty(rows, C, device=src.device, dtype=torch.bfloat16)
    ext().qk_norm_bwd(dout, src, rstd, w, cos, sin, dsrc, dw_acc, L)
    return dsrc
