"""RMSNorm with the adaLN modulation fused in (forward and backward), and the head's LayerNorm.

Forward  h = bf16( w * x * rstd * (1 + scale[g]) + shift[g] ),  rstd = 1 / sqrt(mean(x^2) + eps),  g = row // rows_per_group
Backward with u = w * x * rstd:
    d_shift[g] = sum_rows dh          d_scale[g] = sum_rows dh * u           du = dh * (1 + scale[g])
    d_w        = sum_all_rows du * x * rstd                                    dxn = du * w
    dx         = rstd * (dxn - x * rstd * mean(dxn * x * rstd)) (+ d_residual)
Column sums are deterministic: fixed-order partials per chunk of rows, then a fixed-order reduction.

Reference sites: RMSNorm (baselines/PixelGen/src/models/layers/rmsnorm.py:5-20, fp32 math cast back) composed with
`modulate` (JiT_T2I.py:75-76) in FlattenDiTBlock/TextRefineBlock (JiT_T2I.py:201-210, 279-293), and the Triton fused
norm of the reference's lever K (baselines/PixelGen/src/models/layers/fused_norm.py:64-140), which does the same sums.
"""
import torch

from .._ext import ext
from .elementwise import Segments, _rows


def rms_mod_fwd(x, w, shift=None, scale=None, rows_per_group=1, eps=1e-6):
    """x [M, C] bf16, w [C] fp32, shift/scale [G, C] bf16 views (row stride free) or None.
    Returns (h [M, C] bf16, rstd [M] fp32)."""
    M, C = x.shape
    if not x.is_cuda:
        xf = x.float()
        rstd = torch.rsqrt(xf.pow(2).mean(-1) + eps)
        u = w.float() * xf * rstd[:, None]
        if scale is not None:
            sc = _rows(rows_per_group, scale.float(), M)
            sh = _rows(rows_per_group, shift.float(), M)
            u = u * (1 + sc) + sh
        return u.to(torch.bfloat16), rstd
    h = torch.empty_like(x)
    rstd = torch.empty(M, device=x.device, dtype=torch.float32)
    if isinstance(rows_per_group, Segments):
        ext().rms_mod_fwd(x, w, shift, scale, h, rstd, 1, eps, rows_per_group.seg)
    else:
        ext().rms_mod_fwd(x, w, shift, scale, h, rstd, rows_per_group, eps, None)
    return h, rstd


def rms_mod_fwd_mx(x, w, shift=None, scale=None, rows_per_group=1, eps=1e-6):
    """rms_mod_fwd that also returns h's MXFP8 copy (ops.mx.MX) from the same kernel: (h, rstd, hq). C % 128 == 0."""
    from . import mx
    if not x.is_cuda:
        h, rstd = rms_mod_fwd(x, w, shift, scale, rows_per_group, eps)
        return h, rstd, mx.quant(h)
    M, C = x.shape
    h = torch.empty_like(x)
    rstd = torch.empty(M, device=x.device, dtype=torch.float32)
    q = torch.empty(M, C, device=x.device, dtype=torch.uint8)
    rp = mx.rows_pad(M)
    shape = (rp // 128, C // 128, 512)
    if rp == M:
        sf = torch.empty(shape, device=x.device, dtype=torch.uint8)
    else:  # rows past M (up to the 256-row padding) keep scale 1
        sf = torch.full(shape, 127, device=x.device, dtype=torch.uint8)
    ext().rms_mod_fwd_mx(x, w, shift, scale, h, rstd, q, sf, rows_per_group, eps)
    return h, rstd, mx.MX(q, sf)


def rms_mod_bwd(dh, x, rstd, w, scale=None, rows_per_group=1, dres=None, dw_acc=None, dshift=None, dscale=None):
    """Backward of rms_mod_fwd. Returns dx [M, C] bf16 (plus dres when given).
    dw_acc [C] fp32: d_w is added into it. dshift/dscale [G, C] fp32 views: overwritten (None: not computed).
    rows_per_group may be a Segments (packed rows): rows of no sample then get dx = 0 and add nothing to d_w."""
    M, C = x.shape
    seg = rows_per_group if isinstance(rows_per_group, Segments) else None
    if not x.is_cuda:
        xf, dhf = x.float(), dh.float()
        if seg is not None:
            dhf = dhf * seg.owned(M, dhf.device)[:, None].float()
        xn = xf * rstd[:, None]
        u = w.float() * xn
        if scale is not None:
            G = scale.shape[0]
            sc = _rows(rows_per_group, scale.float(), M)
            du = dhf * (1 + sc)
            if dshift is not None:
                if seg is not None:
                    dshift[:seg.groups].copy_(seg.sum_rows(dhf))
                else:
                    dshift.copy_(dhf.view(G, rows_per_group, C).sum(1))
            if dscale is not None:
                if seg is not None:
                    dscale[:seg.groups].copy_(seg.sum_rows(dhf * u))
                else:
                    dscale.copy_((dhf * u).view(G, rows_per_group, C).sum(1))
        else:
            du = dhf
        if dw_acc is not None:
            dw_acc.add_((du * xn).sum(0))
        dxn = du * w.float()
        dx = rstd[:, None] * (dxn - xn * (dxn * xn).mean(-1, keepdim=True))
        if dres is not None:
            dx = dx + dres.float()
        if seg is not None:
            dx = dx * seg.owned(M, dx.device)[:, None].float()
        return dx.to(torch.bfloat16)
    if seg is not None:
        dx = torch.zeros_like(x)  # rows of no sample keep a zero gradient
        ext().rms_mod_bwd(dh, x, rstd, w, scale, dres, dx, dw_acc, dshift, dscale, 1, seg.cu, seg.max_rows)
        return dx
    dx = torch.empty_like(x)
    ext().rms_mod_bwd(dh, x, rstd, w, scale, dres, dx, dw_acc, dshift, dscale, rows_per_group, None, 0)
    return dx


def layernorm_fwd(x, eps=1e-6):
    """LayerNorm without affine parameters (the head's norm_final, JiT_T2I.py:345-357): fp32 statistics.
    x [M, C] bf16 -> (h [M, C] bf16, mean [M], rstd [M])."""
    if not x.is_cuda:
        xf = x.float()
        mu = xf.mean(-1)
        var = (xf - mu[:, None]).pow(2).mean(-1)
        rstd = torch.rsqrt(var + eps)
        return ((xf - mu[:, None]) * rstd[:, None]).to(torch.bfloat16), mu, rstd
    M, C = x.shape
    h = torch.empty_like(x)
    mu = torch.empty(M, device=x.device, dtype=torch.float32)
    rstd = torch.empty(M, device=x.device, dtype=torch.float32)
    ext().layernorm_fwd(x, h, mu, rstd, eps)
    return h, mu, rstd


def layernorm_bwd(dh, x, mu, rstd):
    """dx = rstd * (dh - mean(dh) - xhat * mean(dh * xhat)) for LayerNorm without affine."""
    if not x.is_cuda:
        xh = (x.float() - mu[:, None]) * rstd[:, None]
        d = dh.float()
        dx = rstd[:, None] * (d - d.mean(-1, keepdim=True) - xh * (d * xh).mean(-1, keepdim=True))
        return dx.to(torch.bfloat16)
    dx = torch.empty_like(x)
    ext().layernorm_bwd(dh, x, mu, rstd, dx)
    return dx
