"""JiT-T2I, the pixel-space text-to-image diffusion transformer, on the framework's fused ops.

Same architecture, initialisation and parameter names (state-dict keys) as the reference's
baselines/PixelGen/src/models/transformer/JiT_T2I.py:359-525, so its checkpoints load strictly:
  x_embedder.proj1/proj2 (bottleneck patch embed), t_embedder.mlp.{0,2}, y_embedder.{proj,norm}, pos_embed (fixed
  sin-cos), y_pos_embedding, text_refine_blocks.* (adaLN text self-attention blocks), blocks.* (adaLN image blocks with
  joint attention over [image ; caption] keys), final_layer.linear (after a LayerNorm without affine).

Execution: every transformer block is one torch.autograd.Function whose forward runs the fused kernels (tcgen05 GEMMs
with fused epilogues, RMSNorm+modulate, q/k norm + RoPE, masked attention) and whose backward is written out by hand.
Weight gradients go straight into each parameter's fp32 `.grad` (which nano_gpic_b200.parallel.flat makes views of one
flat buffer), accumulated across micro-batches by the GEMM epilogue; only activation gradients flow through autograd.
Compute weights are bf16 shadows of the fp32 master weights (refreshed after every optimizer step).

Inputs: x [B, 3, H, W], t [B], y [B, T, txt_embed_dim] caption features, y_mask [B, T] bool (left-aligned, True = a
real token) or None (all T tokens real). The caption-length handling is the reference's masked path (option B): padded
caption keys are masked out of every attention. Or packed captions (the reference's lever E): y [S, txt_embed_dim]
with y_pack; the text blocks and the caption projections then run on the S packed rows (`Packing`).
"""
import math
import os

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import attention as A
from ..ops import elementwise as E
from ..ops import gemm as G
from ..ops import mx as MXO
from ..ops import norm as NR
from ..ops import qk as QK
from .layers import Linear, RMSNorm, rope_tables, sincos_pos_embed, timestep_freq

BF16 = torch.bfloat16


# ------------------------------------------------------------------------------------------------------ weights
def w16(lin_or_param):
    """bf16 compute copy of a weight: the flat bf16 shadow when the model has one, else a cast."""
    p = lin_or_param.weight if isinstance(lin_or_param, nn.Module) else lin_or_param
    s = getattr(p, "_bf16", None)
    if s is not None:
        return s
    return p.detach().to(BF16)


def f32(p):
    """fp32 master value of a (small) parameter, without autograd."""
    return p.detach()


def grad_of(p):
    """The parameter's fp32 gradient buffer (created on first use when the model has no flat store)."""
    if p.grad is None:
        p.grad = torch.zeros_like(p, dtype=torch.float32)
    return p.grad


def _wgrad(dy, x, p):
    G.linear_wgrad(dy, x, out=grad_of(p), accumulate=True)


def _mx_weights(blk):
    """MXFP8 copies of an image block's forward GEMM weights (qkv_x, proj, w12, w3) and, with the MLP backward in FP8
    (fp8 "mx2"), of the transposed MLP weights its dgrads read (w3t [H, C], w12t [C, 2H]); made from the bf16 compute
    weights once per weight version (JiT_T2I.weights_changed() after every optimizer step or load)."""
    ver = getattr(blk, "_wver", 0)
    c = getattr(blk, "_mxw", None)
    if c is None or c[0] != ver:
        a = blk.attn
        d = {"qkv_x": MXO.quant(w16(a.qkv_x)), "proj": MXO.quant(w16(a.proj)),
             "w12": MXO.quant(w16(blk.mlp.w12)), "w3": MXO.quant(w16(blk.mlp.w3))}
        if getattr(blk, "_fp8_bwd", False):
            d["w3t"] = MXO.quant(w16(blk.mlp.w3).t().contiguous())
            d["w12t"] = MXO.quant(w16(blk.mlp.w12).t().contiguous())
        c = (ver, d)
        blk._mxw = c
    return c[1]


def _bias_grad(dy, p):
    E.colsum(dy, grad_of(p), accumulate=True)


# ------------------------------------------------------------------------------------------------------ modules
class SwiGLU(nn.Module):
    """w12: C -> 2 * hidden (no bias), w3: hidden -> C (no bias); reference layers/swiglu.py:4-24."""

    def __init__(self, dim, hidden):
        super().__init__()
        self.w12 = Linear(dim, 2 * hidden, bias=False)
        self.w3 = Linear(hidden, dim, bias=False)


class Attention(nn.Module):
    """Image-block attention parameters (reference JiT_T2I.py:114-138)."""

    def __init__(self, dim, num_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.qkv_x = Linear(dim, 3 * dim, bias=False)
        self.kv_y = Linear(dim, 2 * dim, bias=False)
        self.q_norm = RMSNorm(self.head_dim)
        self.k_norm = RMSNorm(self.head_dim)
        self.proj = Linear(dim, dim, bias=True)


class TextRefineAttention(nn.Module):
    """Text-block attention parameters (reference JiT_T2I.py:212-232)."""

    def __init__(self, dim, num_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.qkv = Linear(dim, 3 * dim, bias=False)
        self.q_norm = RMSNorm(self.head_dim)
        self.k_norm = RMSNorm(self.head_dim)
        self.proj = Linear(dim, dim, bias=True)


class AdaLN(nn.Module):
    """`adaLN_modulation = nn.Sequential(nn.Linear(C, 6C))`: keeps the `.0.` in the parameter names."""

    def __init__(self, dim):
        super().__init__()
        self.add_module("0", Linear(dim, 6 * dim, bias=True))

    @property
    def lin(self):
        return self._modules["0"]


class FlattenDiTBlock(nn.Module):
    def __init__(self, hidden, heads, mlp_ratio=4):
        super().__init__()
        self.norm1 = RMSNorm(hidden)
        self.attn = Attention(hidden, heads)
        self.norm2 = RMSNorm(hidden)
        self.mlp = SwiGLU(hidden, int(hidden * mlp_ratio))
        self.adaLN_modulation = AdaLN(hidden)


class TextRefineBlock(nn.Module):
    def __init__(self, hidden, heads, mlp_ratio=4):
        super().__init__()
        self.norm1 = RMSNorm(hidden)
        self.attn = TextRefineAttention(hidden, heads)
        self.norm2 = RMSNorm(hidden)
        self.mlp = SwiGLU(hidden, int(hidden * mlp_ratio))
        self.adaLN_modulation = AdaLN(hidden)


class BottleneckEmbed(nn.Module):
    def __init__(self, in_chans, embed_dim, bottleneck_dim):
        super().__init__()
        self.proj1 = Linear(in_chans, bottleneck_dim, bias=False)
        self.proj2 = Linear(bottleneck_dim, embed_dim, bias=True)


class TimestepEmbedder(nn.Module):
    """mlp = Linear(256, C), SiLU, Linear(C, C) (reference layers/time_embed.py:5-29, max_period 10); both Linears on
    the tcgen05 GEMM with the bias in the epilogue (`_TimeEmbedFn`), weight gradients into the fp32 .grad buffers."""

    def __init__(self, hidden, freq_dim=256):
        super().__init__()
        self.freq_dim = freq_dim
        self.mlp = nn.Sequential(nn.Linear(freq_dim, hidden, bias=True), nn.SiLU(), nn.Linear(hidden, hidden, bias=True))

    def forward(self, t):
        f = timestep_freq(t.view(-1), self.freq_dim).to(BF16)
        l0, l2 = self.mlp[0], self.mlp[2]
        return _TimeEmbedFn.apply(f, l0.weight, l0, l2)


class CaptionEmbed(nn.Module):
    """Linear(txt_embed_dim, C) + RMSNorm(C) (reference layers/patch_embed.py:6-21)."""

    def __init__(self, in_dim, dim):
        super().__init__()
        self.proj = Linear(in_dim, dim, bias=True)
        self.norm = RMSNorm(dim)


class FinalLayer(nn.Module):
    """LayerNorm(C, no affine, eps 1e-6) then Linear(C, patch_dim) (reference JiT_T2I.py:345-357)."""

    def __init__(self, dim, out_dim):
        super().__init__()
        self.linear = Linear(dim, out_dim, bias=True)


# ------------------------------------------------------------------------------------------- block functions
def _stage_hook(hook):
    """hook = (model, n): at the start of a block's backward the first n backward stages (final layer, image blocks
    from the last, text blocks from the last) hold final gradients; tell the data-parallel layer, if it listens."""
    if hook is not None and hook[0]._bwd_hook is not None:
        hook[0]._bwd_hook(hook[1])


class Packing:
    """Packed captions (the reference's y_pack, JiT_T2I.py:54-65): the caption tokens of the batch back to back,
    S rows (the real tokens, then dummy rows up to a bucketed count). Built once per forward from y_pack:
      segs  Segments: row -> its sample's modulation row (dummy rows -> a zero row B), sample b owns rows
            [cu[b], cu[b + 1]), at most Tp of them
      pidx  [S] int32: the row's place b * Tp + pos in the padded [B, Tp] layout, -1 for a dummy row
      inv   [B * Tp] int32: the packed row of each padded place, -1 for padding
      lens  [B] int32 caption lengths, Tp the padded width (>= the longest caption)
    The text blocks and the caption key/value projections run on the S packed rows; only the attention reads the
    padded layout (gathered in one pass per tensor), as the reference's default text attention does."""

    def __init__(self, y_pack, S, device):
        kmask = y_pack["kmask"]
        B, Tp = kmask.shape
        self.B, self.Tp, self.S = B, Tp, S
        self.lens = y_pack["lens"].to(device=device, dtype=torch.int32)
        cu = y_pack["cu"].to(device=device, dtype=torch.int32).contiguous()
        p = y_pack["pidx"].to(device=device, dtype=torch.int64)
        real = p < B * Tp
        self.pidx = torch.where(real, p, torch.full_like(p, -1)).to(torch.int32).contiguous()
        seg = torch.where(real, torch.div(p, Tp, rounding_mode="floor"), torch.full_like(p, B))
        self.segs = E.Segments(seg.to(torch.int32).contiguous(), cu, Tp)
        inv = torch.full((B * Tp + 1,), -1, dtype=torch.int64, device=device)
        inv.scatter_(0, torch.where(real, p, torch.full_like(p, B * Tp)), torch.arange(S, device=device))
        inv[B * Tp] = -1
        self.inv = inv[:B * Tp].to(torch.int32).contiguous()
        self.pos = y_pack["pos"].to(device=device, dtype=torch.int32).contiguous()

    def to_padded(self, t):
        return E.gather_rows(t, self.inv)

    def to_packed(self, t, out=None):
        return E.gather_rows(t, self.pidx, out)


def _with_zero_row(mod):
    """mod [B, 6C] with a zero row appended: the modulation of the dummy rows of packed captions."""
    return torch.cat([mod, mod.new_zeros(1, mod.shape[1])])


class _TextBlockFn(torch.autograd.Function):
    @staticmethod
    def _run(y, mod, blk, lens, T, pack=None):
        """The block's forward: (output, the activations its backward reads). pack: a Packing (y holds packed rows)
        or None (T rows per sample)."""
        C = y.shape[1]
        a = blk.attn
        n1, n2 = blk.norm1, blk.norm2
        grp = T if pack is None else pack.segs
        h1, r1 = NR.rms_mod_fwd(y, f32(n1.weight), mod[:, 0:C], mod[:, C:2 * C], grp, n1.variance_epsilon)
        qkv = G.linear(h1, w16(a.qkv))
        q, rq = QK.qk_norm_fwd(qkv[:, 0:C], f32(a.q_norm.weight), eps=a.q_norm.variance_epsilon)
        k, rk = QK.qk_norm_fwd(qkv[:, C:2 * C], f32(a.k_norm.weight), eps=a.k_norm.variance_epsilon)
        if pack is None:
            o, lse = A.attn_fwd(q, T, k, qkv[:, 2 * C:], T, lens)
            padded = ()
        else:  # the attention on the padded layout, its output back to the packed rows (dummy rows read zeros)
            qp, kp, vp = pack.to_padded(q), pack.to_padded(k), pack.to_padded(qkv[:, 2 * C:])
            op, lse = A.attn_fwd(qp, pack.Tp, kp, vp, pack.Tp, lens)
            o = pack.to_packed(op)
            padded = (qp, kp, vp, op)
        y2, ya = G.linear_gated_residual(o, w16(a.proj), f32(a.proj.bias), y, mod[:, 2 * C:3 * C], grp)
        h2, r2 = NR.rms_mod_fwd(y2, f32(n2.weight), mod[:, 3 * C:4 * C], mod[:, 4 * C:5 * C], grp, n2.variance_epsilon)
        act, pre = G.swiglu_linear(h2, w16(blk.mlp.w12))
        y3, ym = G.linear_gated_residual(act, w16(blk.mlp.w3), None, y2, mod[:, 5 * C:6 * C], grp)
        return y3, (h1, r1, qkv, q, rq, k, rk, o, lse, y2, ya, h2, r2, act, pre, ym) + padded

    @staticmethod
    def forward(ctx, y, mod, anchor, blk, lens, T, hook=None, pack=None):
        if pack is not None:
            mod = _with_zero_row(mod)
        y3, acts = _TextBlockFn._run(y, mod, blk, lens, T, pack)
        ctx.blk, ctx.T, ctx.hook, ctx.pack = blk, T, hook, pack
        ctx.recompute = getattr(blk, "_recompute", False)
        ctx.save_for_backward(y, mod, lens, *(() if ctx.recompute else acts))
        return y3

    @staticmethod
    def backward(ctx, dy3):
        y, mod, lens, *acts = ctx.saved_tensors
        blk, T, pack = ctx.blk, ctx.T, ctx.pack
        _stage_hook(ctx.hook)
        if ctx.recompute:  # activation checkpointing: rerun the forward from the saved inputs
            acts = _TextBlockFn._run(y, mod, blk, lens, T, pack)[1]
        (h1, r1, qkv, q, rq, k, rk, o, lse, y2, ya, h2, r2, act, pre, ym) = acts[:16]
        grp = T if pack is None else pack.segs
        a = blk.attn
        C = y.shape[1]
        dy3 = dy3.contiguous()
        dmod = torch.empty(mod.shape, device=mod.device, dtype=torch.float32)
        # mlp branch: y3 = y2 + g2 * w3(act)
        dym = E.gate_bwd(dy3, ym, mod[:, 5 * C:6 * C], grp, dgate=dmod[:, 5 * C:6 * C])
        dpre = G.swiglu_dgrad(dym, w16(blk.mlp.w3), pre)
        _wgrad(dym, act, blk.mlp.w3.weight)
        dh2 = G.linear_dgrad(dpre, w16(blk.mlp.w12))
        _wgrad(dpre, h2, blk.mlp.w12.weight)
        dy2 = NR.rms_mod_bwd(dh2, y2, r2, f32(blk.norm2.weight), mod[:, 4 * C:5 * C], grp, dres=dy3,
                             dw_acc=grad_of(blk.norm2.weight), dshift=dmod[:, 3 * C:4 * C],
                             dscale=dmod[:, 4 * C:5 * C])
        # attention branch: y2 = y + g1 * proj(o)
        dya = E.gate_bwd(dy2, ya, mod[:, 2 * C:3 * C], grp, dgate=dmod[:, 2 * C:3 * C], dbias=grad_of(a.proj.bias))
        do = G.linear_dgrad(dya, w16(a.proj))
        _wgrad(dya, o, a.proj.weight)
        dqkv = torch.empty_like(qkv)
        if pack is None:
            dq, dk, _, _, _ = A.attn_bwd(do, q, T, k, qkv[:, 2 * C:], T, lens, o, lse, dv0=dqkv[:, 2 * C:])
        else:
            qp, kp, vp, op = acts[16:]
            dvp = torch.empty_like(vp)
            dqp, dkp, _, _, _ = A.attn_bwd(pack.to_padded(do), qp, pack.Tp, kp, vp, pack.Tp, lens, op, lse, dv0=dvp)
            pack.to_packed(dvp, out=dqkv[:, 2 * C:])
            dq, dk = pack.to_packed(dqp), pack.to_packed(dkp)
        QK.qk_norm_bwd(dq, qkv[:, 0:C], rq, f32(a.q_norm.weight), dsrc=dqkv[:, 0:C], dw_acc=grad_of(a.q_norm.weight))
        QK.qk_norm_bwd(dk, qkv[:, C:2 * C], rk, f32(a.k_norm.weight), dsrc=dqkv[:, C:2 * C],
                       dw_acc=grad_of(a.k_norm.weight))
        dh1 = G.linear_dgrad(dqkv, w16(a.qkv))
        _wgrad(dqkv, h1, a.qkv.weight)
        dy = NR.rms_mod_bwd(dh1, y, r1, f32(blk.norm1.weight), mod[:, C:2 * C], grp, dres=dy2,
                            dw_acc=grad_of(blk.norm1.weight), dshift=dmod[:, 0:C], dscale=dmod[:, C:2 * C])
        if pack is not None:
            dmod = dmod[:pack.B]  # the dummy rows' zero modulation row is no input
        return dy, dmod.to(BF16), None, None, None, None, None, None


class _ImageBlockFn(torch.autograd.Function):
    @staticmethod
    def _run(x, yt, mod, blk, lens, L, T, cos, sin, pack=None):
        """The block's forward: (output, the activations its backward reads). pack: a Packing (yt holds packed caption
        rows) or None (T rows per sample)."""
        C = x.shape[1]
        a = blk.attn
        n1, n2 = blk.norm1, blk.norm2
        # fp8 == "mx": the four big forward GEMMs read MXFP8 operands (reference fp8_native.py, phase 1); the saved
        # activations and the whole backward stay bf16
        mxw = _mx_weights(blk) if getattr(blk, "_fp8", False) else None
        if mxw is None:
            h1, r1 = NR.rms_mod_fwd(x, f32(n1.weight), mod[:, 0:C], mod[:, C:2 * C], L, n1.variance_epsilon)
            qkv = G.linear(h1, w16(a.qkv_x))
        else:  # the norm kernel also writes h1's MXFP8 copy
            h1, r1, h1q = NR.rms_mod_fwd_mx(x, f32(n1.weight), mod[:, 0:C], mod[:, C:2 * C], L, n1.variance_epsilon)
            qkv = MXO.linear(h1q, mxw["qkv_x"])
        kvy = G.linear(yt, w16(a.kv_y))
        q, rq = QK.qk_norm_fwd(qkv[:, 0:C], f32(a.q_norm.weight), cos, sin, L, a.q_norm.variance_epsilon)
        kx, rkx = QK.qk_norm_fwd(qkv[:, C:2 * C], f32(a.k_norm.weight), cos, sin, L, a.k_norm.variance_epsilon)
        ky, rky = QK.qk_norm_fwd(kvy[:, 0:C], f32(a.k_norm.weight), eps=a.k_norm.variance_epsilon)
        if pack is None:
            o, lse = A.attn_fwd(q, L, kx, qkv[:, 2 * C:], L, L, ky, kvy[:, C:], T, lens)
            padded = ()
        else:  # packed caption keys/values placed in the padded [B, Tp] layout the attention reads
            kyp, vyp = pack.to_padded(ky), pack.to_padded(kvy[:, C:])
            o, lse = A.attn_fwd(q, L, kx, qkv[:, 2 * C:], L, L, kyp, vyp, pack.Tp, lens)
            padded = (kyp, vyp)
        if mxw is None:
            x2, ya = G.linear_gated_residual(o, w16(a.proj), f32(a.proj.bias), x, mod[:, 2 * C:3 * C], L)
        else:
            x2, ya = MXO.linear_gated_residual(MXO.quant(o), mxw["proj"], f32(a.proj.bias), x, mod[:, 2 * C:3 * C], L)
        if mxw is None:
            h2, r2 = NR.rms_mod_fwd(x2, f32(n2.weight), mod[:, 3 * C:4 * C], mod[:, 4 * C:5 * C], L,
                                    n2.variance_epsilon)
            act, pre = G.swiglu_linear(h2, w16(blk.mlp.w12))
            x3, ym = G.linear_gated_residual(act, w16(blk.mlp.w3), None, x2, mod[:, 5 * C:6 * C], L)
        else:
            h2, r2, h2q = NR.rms_mod_fwd_mx(x2, f32(n2.weight), mod[:, 3 * C:4 * C], mod[:, 4 * C:5 * C], L,
                                            n2.variance_epsilon)
            act, pre, actq = MXO.swiglu_linear(h2q, mxw["w12"], quant_act=True)  # act's MX copy from the epilogue
            x3, ym = MXO.linear_gated_residual(actq, mxw["w3"], None, x2, mod[:, 5 * C:6 * C], L)
        return x3, (h1, r1, qkv, kvy, q, rq, kx, rkx, ky, rky, o, lse, x2, ya, h2, r2, act, pre, ym) + padded

    @staticmethod
    def forward(ctx, x, yt, mod, anchor, blk, lens, L, T, cos, sin, hook=None, pack=None):
        x3, acts = _ImageBlockFn._run(x, yt, mod, blk, lens, L, T, cos, sin, pack)
        ctx.blk, ctx.L, ctx.T, ctx.hook, ctx.pack = blk, L, T, hook, pack
        ctx.recompute = getattr(blk, "_recompute", False)
        ctx.save_for_backward(x, yt, mod, lens, cos, sin, *(() if ctx.recompute else acts))
        return x3

    @staticmethod
    def backward(ctx, dx3):
        x, yt, mod, lens, cos, sin, *acts = ctx.saved_tensors
        blk, L, T, pack = ctx.blk, ctx.L, ctx.T, ctx.pack
        _stage_hook(ctx.hook)
        if ctx.recompute:  # activation checkpointing: rerun the forward from the saved inputs
            acts = _ImageBlockFn._run(x, yt, mod, blk, lens, L, T, cos, sin, pack)[1]
        (h1, r1, qkv, kvy, q, rq, kx, rkx, ky, rky, o, lse, x2, ya, h2, r2, act, pre, ym) = acts[:19]
        a = blk.attn
        C = x.shape[1]
        dx3 = dx3.contiguous()
        dmod = torch.empty(mod.shape, device=mod.device, dtype=torch.float32)
        dym = E.gate_bwd(dx3, ym, mod[:, 5 * C:6 * C], L, dgate=dmod[:, 5 * C:6 * C])
        if getattr(blk, "_fp8_bwd", False):
            # the MLP's dgrads in MXFP8 (the reference's phase 2, fp8_native.py:236-266): dy's MX copy, the w3 dgrad
            # with the SwiGLU backward in its epilogue writing d(pre) in bf16 (w12's weight gradient) and in MXFP8
            # (w12's dgrad); weight gradients stay bf16
            mxw = _mx_weights(blk)
            dpre, dpreq = MXO.swiglu_dgrad(MXO.quant(dym), mxw["w3t"], pre, quant_out=True)
            dh2 = MXO.linear(dpreq, mxw["w12t"])
        else:
            dpre = G.swiglu_dgrad(dym, w16(blk.mlp.w3), pre)
            dh2 = G.linear_dgrad(dpre, w16(blk.mlp.w12))
        _wgrad(dym, act, blk.mlp.w3.weight)
        _wgrad(dpre, h2, blk.mlp.w12.weight)
        dx2 = NR.rms_mod_bwd(dh2, x2, r2, f32(blk.norm2.weight), mod[:, 4 * C:5 * C], L, dres=dx3,
                             dw_acc=grad_of(blk.norm2.weight), dshift=dmod[:, 3 * C:4 * C],
                             dscale=dmod[:, 4 * C:5 * C])
        dya = E.gate_bwd(dx2, ya, mod[:, 2 * C:3 * C], L, dgate=dmod[:, 2 * C:3 * C], dbias=grad_of(a.proj.bias))
        do = G.linear_dgrad(dya, w16(a.proj))
        _wgrad(dya, o, a.proj.weight)
        dqkv = torch.empty_like(qkv)
        dkvy = torch.empty_like(kvy)
        if pack is None:
            dq, dkx, _, dky, _ = A.attn_bwd(do, q, L, kx, qkv[:, 2 * C:], L, L, o, lse, ky, kvy[:, C:], T, lens,
                                            dv0=dqkv[:, 2 * C:], dv1=dkvy[:, C:])
        else:
            kyp, vyp = acts[19:]
            dvyp = torch.empty_like(vyp)
            dq, dkx, _, dkyp, _ = A.attn_bwd(do, q, L, kx, qkv[:, 2 * C:], L, L, o, lse, kyp, vyp, pack.Tp, lens,
                                             dv0=dqkv[:, 2 * C:], dv1=dvyp)
            pack.to_packed(dvyp, out=dkvy[:, C:])
            dky = pack.to_packed(dkyp)
        QK.qk_norm_bwd(dq, qkv[:, 0:C], rq, f32(a.q_norm.weight), cos, sin, L, dsrc=dqkv[:, 0:C],
                       dw_acc=grad_of(a.q_norm.weight))
        dwk = grad_of(a.k_norm.weight)
        QK.qk_norm_bwd(dkx, qkv[:, C:2 * C], rkx, f32(a.k_norm.weight), cos, sin, L, dsrc=dqkv[:, C:2 * C], dw_acc=dwk)
        QK.qk_norm_bwd(dky, kvy[:, 0:C], rky, f32(a.k_norm.weight), dsrc=dkvy[:, 0:C], dw_acc=dwk)
        dh1 = G.linear_dgrad(dqkv, w16(a.qkv_x))
        _wgrad(dqkv, h1, a.qkv_x.weight)
        dyt = G.linear_dgrad(dkvy, w16(a.kv_y))
        _wgrad(dkvy, yt, a.kv_y.weight)
        dx = NR.rms_mod_bwd(dh1, x, r1, f32(blk.norm1.weight), mod[:, C:2 * C], L, dres=dx2,
                            dw_acc=grad_of(blk.norm1.weight), dshift=dmod[:, 0:C], dscale=dmod[:, C:2 * C])
        return dx, dyt, dmod.to(BF16), None, None, None, None, None, None, None, None, None


class _ModFn(torch.autograd.Function):
    """adaLN modulation mod = c W^T + b on the tcgen05 GEMM (bias in the epilogue) from the bf16 weight shadow (the
    reference's autocast Linear(C, 6C)); W and b gradients into the fp32 .grad buffers, dc = dmod W."""

    @staticmethod
    def forward(ctx, c16, anchor, lin):
        ctx.lin = lin
        ctx.save_for_backward(c16)
        return G.linear(c16.contiguous(), w16(lin), f32(lin.bias))

    @staticmethod
    def backward(ctx, dmod):
        (c16,) = ctx.saved_tensors
        lin = ctx.lin
        dmod = dmod.to(BF16).contiguous()
        _wgrad(dmod, c16, lin.weight)
        _bias_grad(dmod, lin.bias)
        return G.linear_dgrad(dmod, w16(lin)), None, None


class _TimeEmbedFn(torch.autograd.Function):
    """t_emb = W2 silu(W1 f + b1) + b2 for the sinusoidal features f [B, 256] bf16: two GEMMs with bias epilogues,
    bf16 activations as under the reference's autocast; the weight and bias gradients go into .grad, no gradient
    flows to f (the timesteps are data)."""

    @staticmethod
    def forward(ctx, f, anchor, l0, l2):
        h = G.linear(f, w16(l0), f32(l0.bias))
        s = F.silu(h)
        ctx.l0, ctx.l2 = l0, l2
        ctx.save_for_backward(f, h, s)
        return G.linear(s, w16(l2), f32(l2.bias))

    @staticmethod
    def backward(ctx, dt):
        f, h, s = ctx.saved_tensors
        l0, l2 = ctx.l0, ctx.l2
        dt = dt.to(BF16).contiguous()
        _wgrad(dt, s, l2.weight)
        _bias_grad(dt, l2.bias)
        ds = G.linear_dgrad(dt, w16(l2)).float()
        sig = torch.sigmoid(h.float())
        dh = (ds * sig * (1 + h.float() * (1 - sig))).to(BF16)
        _wgrad(dh, f, l0.weight)
        _bias_grad(dh, l0.bias)
        return None, None, None, None


class _LinearFn(torch.autograd.Function):
    """y = x w^T + b on the tcgen05 GEMM; weight/bias gradients into the parameters' fp32 .grad."""

    @staticmethod
    def forward(ctx, x, anchor, lin, need_dx):
        ctx.lin, ctx.need_dx = lin, need_dx
        ctx.save_for_backward(x)
        return G.linear(x, w16(lin), f32(lin.bias) if lin.bias is not None else None)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        lin = ctx.lin
        dy = dy.contiguous()
        _wgrad(dy, x, lin.weight)
        if lin.bias is not None:
            _bias_grad(dy, lin.bias)
        dx = G.linear_dgrad(dy, w16(lin)) if ctx.need_dx else None
        return dx, None, None, None


class _RMSFn(torch.autograd.Function):
    """Plain RMSNorm (the caption embed's norm) with its weight gradient into .grad."""

    @staticmethod
    def forward(ctx, x, anchor, norm):
        h, r = NR.rms_mod_fwd(x, f32(norm.weight), eps=norm.variance_epsilon)
        ctx.norm = norm
        ctx.save_for_backward(x, r)
        return h

    @staticmethod
    def backward(ctx, dh):
        x, r = ctx.saved_tensors
        return NR.rms_mod_bwd(dh.contiguous(), x, r, f32(ctx.norm.weight), dw_acc=grad_of(ctx.norm.weight)), None, None


class _AddRowsFn(torch.autograd.Function):
    """bf16(a + table[row % period]); the table's gradient (summed over periods) goes into `param.grad` when given."""

    @staticmethod
    def forward(ctx, a, anchor, table, period, param):
        ctx.period, ctx.param = period, param
        return E.add_rows(a, table, period)

    @staticmethod
    def backward(ctx, d):
        if ctx.param is not None:
            P = ctx.period
            g = grad_of(ctx.param)
            Cd = d.shape[-1]
            E.colsum(d.reshape(-1, P * Cd), g.view(-1)[:P * Cd], accumulate=True)
        return d, None, None, None, None


class _AddPosFn(torch.autograd.Function):
    """Packed captions: bf16(a + table[pos[row]]) (the reference's y_pos_embedding[0].index_select(0, pos)); the
    table's gradient sums each position over the real rows (dummy rows add nothing), through the padded layout, in a
    fixed order."""

    @staticmethod
    def forward(ctx, a, anchor, table, pack, param):
        ctx.pack, ctx.param = pack, param
        return a + E.gather_rows(table, pack.pos)

    @staticmethod
    def backward(ctx, d):
        pack, param = ctx.pack, ctx.param
        d = d.contiguous()
        if param is not None:
            Cd = d.shape[-1]
            P = pack.Tp
            dp = pack.to_padded(d)  # [B * Tp, C], zeros where no token
            E.colsum(dp.reshape(-1, P * Cd), grad_of(param).view(-1)[:P * Cd], accumulate=True)
        return d, None, None, None, None


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, eps):
        h, mu, r = NR.layernorm_fwd(x, eps)
        ctx.save_for_backward(x, mu, r)
        return h

    @staticmethod
    def backward(ctx, dh):
        x, mu, r = ctx.saved_tensors
        return NR.layernorm_bwd(dh.contiguous(), x, mu, r), None


class _UnpatchifyFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tok, shape, p):
        ctx.p = p
        return E.unpatchify(tok, *shape, p)

    @staticmethod
    def backward(ctx, d):
        return E.patchify(d.contiguous(), ctx.p), None, None


# ---------------------------------------------------------------------------------------------------------- model
class JiT_T2I(nn.Module):
    def __init__(self, input_size=256, in_channels=4, num_groups=12, hidden_size=1152, num_blocks=18,
                 num_text_blocks=4, patch_size=2, txt_embed_dim=1024, txt_max_length=100, bottleneck_dim=256,
                 weight_path=None, load_ema=False, fp8=None, recompute=None):
        super().__init__()
        assert hidden_size % num_groups == 0 and hidden_size // num_groups == 64, "head dim 64 expected"
        self.in_channels = self.out_channels = in_channels
        self.hidden_size, self.num_groups = hidden_size, num_groups
        self.num_blocks, self.num_text_blocks = num_blocks, num_text_blocks
        self.patch_size, self.input_size = patch_size, input_size
        self.txt_embed_dim, self.txt_max_length = txt_embed_dim, txt_max_length
        self.weight_path, self.load_ema = weight_path, load_ema
        patch_dim = in_channels * patch_size ** 2
        self.x_embedder = BottleneckEmbed(patch_dim, hidden_size, bottleneck_dim)
        self.t_embedder = TimestepEmbedder(hidden_size)
        self.y_embedder = CaptionEmbed(txt_embed_dim, hidden_size)
        self.num_patches = (input_size // patch_size) ** 2
        self.pos_embed = nn.Parameter(torch.zeros(1, self.num_patches, hidden_size), requires_grad=False)
        self.y_pos_embedding = nn.Parameter(torch.randn(1, txt_max_length, hidden_size) * 0.02)
        self.blocks = nn.ModuleList([FlattenDiTBlock(hidden_size, num_groups) for _ in range(num_blocks)])
        self.text_refine_blocks = nn.ModuleList([TextRefineBlock(hidden_size, num_groups)
                                                 for _ in range(num_text_blocks)])
        self.final_layer = FinalLayer(hidden_size, patch_dim)
        self.initialize_weights()
        for p in self.t_embedder.parameters():  # small and read by every micro-batch first: replicated under sharding
            p._replicate = True
        self._rope = {}
        self._bwd_hook = None  # set by the data-parallel layer around the last micro-batch's backward
        if fp8 is None and os.environ.get("GPIC_MFU_FP8", "") not in ("", "0", "off"):
            # the reference's switch (GPIC_MFU_FP8=native / native2) selects this package's MXFP8 GEMMs
            fp8 = "mx2" if os.environ["GPIC_MFU_FP8"] == "native2" else "mx"
        self.set_fp8(fp8)
        self.set_recompute(recompute)

    # -------------------------------------------------------------------------------------- activation memory
    def set_recompute(self, mode):
        """Activation checkpointing (no counterpart in the reference): None keeps every block's activations for the
        backward; "image" keeps only the image blocks' inputs and reruns their forward in the backward; "all" does the
        same for the text blocks too. Trades one extra forward of those blocks for their activation memory."""
        assert mode in (None, "image", "all"), f"recompute mode {mode!r}: None, 'image' or 'all'"
        self.recompute = mode
        for blk in self.blocks:
            blk._recompute = mode is not None
        for blk in self.text_refine_blocks:
            blk._recompute = mode == "all"

    # ------------------------------------------------------------------------------------------------- fp8
    def set_fp8(self, mode):
        """None: bf16 GEMMs everywhere. "mx": the image blocks' qkv_x / proj / w12 / w3 forward GEMMs in MXFP8 (the
        reference's GPIC_MFU_FP8=native, phase 1). "mx2": also the MLP's two dgrads (w3, w12) in MXFP8 (native2, its
        phase 2)."""
        assert mode in (None, "mx", "mx2"), f"fp8 mode {mode!r}: None, 'mx' or 'mx2'"
        self.fp8 = mode
        for blk in self.blocks:
            blk._fp8 = mode in ("mx", "mx2")
            blk._fp8_bwd = mode == "mx2"
            blk._mxw = None
        self.weights_changed()

    def weights_changed(self):
        """Marks the weights as updated (after an optimizer step or a load): derived copies are rebuilt lazily."""
        self._wver = getattr(self, "_wver", 0) + 1
        for blk in self.blocks:
            blk._wver = self._wver

    # ------------------------------------------------------------------------------------------------- init
    def initialize_weights(self):
        """Reference JiT_T2I.initialize_weights (JiT_T2I.py:426-461): Xavier-uniform Linears with zero biases, the
        fixed sin-cos pos_embed, N(0, 0.02) time-MLP weights, zero adaLN and zero final linear."""
        for m in self.modules():
            if isinstance(m, (Linear, nn.Linear)):
                nn.init.xavier_uniform_(m.weight)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
        grid = int(self.num_patches ** 0.5)
        self.pos_embed.data.copy_(sincos_pos_embed(self.hidden_size, grid).unsqueeze(0))
        nn.init.xavier_uniform_(self.x_embedder.proj1.weight)
        nn.init.xavier_uniform_(self.x_embedder.proj2.weight)
        nn.init.zeros_(self.x_embedder.proj2.bias)
        nn.init.normal_(self.t_embedder.mlp[0].weight, std=0.02)
        nn.init.normal_(self.t_embedder.mlp[2].weight, std=0.02)
        for blk in list(self.blocks) + list(self.text_refine_blocks):
            nn.init.zeros_(blk.adaLN_modulation.lin.weight)
            nn.init.zeros_(blk.adaLN_modulation.lin.bias)
        nn.init.zeros_(self.final_layer.linear.weight)
        nn.init.zeros_(self.final_layer.linear.bias)

    def rope(self, device):
        key = str(device)
        if key not in self._rope:
            g = self.input_size // self.patch_size
            self._rope[key] = rope_tables(self.hidden_size // self.num_groups, g, g, device=device)
        return self._rope[key]

    # ---------------------------------------------------------------------------------------------- forward
    def _caption_lens(self, y, y_mask):
        B, T = y.shape[:2]
        if y_mask is None:
            return torch.full((B,), T, dtype=torch.int32, device=y.device)
        return y_mask.sum(1, dtype=torch.int32)

    def forward_tokens(self, x_tok, t, y, y_mask=None, y_pack=None):
        """x_tok: [B*N, patch_dim] bf16 patch tokens -> predicted clean-image tokens [B*N, patch_dim] bf16.
        y: [B, T, txt_embed_dim] with y_mask, or packed [S, txt_embed_dim] with y_pack (the reference's lever E
        format: lens, cu, pidx, kmask, pos; JiT_T2I.py:54-65,478-496 there)."""
        N, C = self.num_patches, self.hidden_size
        cos, sin = self.rope(x_tok.device)
        # condition: c = silu(t_embedder(t))  [B, C]
        c = F.silu(self.t_embedder(t.view(-1)))
        # caption tokens: RMSNorm(Linear(y)) + y_pos_embedding[position]
        pack = None
        if y_pack is not None:
            pack = Packing(y_pack, y.shape[0], x_tok.device)
            T, lens = pack.Tp, pack.lens
            yt = y.to(BF16).contiguous()
        else:
            B, T = y.shape[:2]
            lens = self._caption_lens(y, y_mask)
            yt = y.reshape(B * T, -1).to(BF16)
        yt = _LinearFn.apply(yt, self.y_embedder.proj.weight, self.y_embedder.proj, False)
        yt = _RMSFn.apply(yt, self.y_embedder.norm.weight, self.y_embedder.norm)
        if pack is None:
            yt = _AddRowsFn.apply(yt, self.y_pos_embedding, w16(self.y_pos_embedding)[0, :T], T, self.y_pos_embedding)
        else:
            yt = _AddPosFn.apply(yt, self.y_pos_embedding, w16(self.y_pos_embedding)[0], pack, self.y_pos_embedding)
        nb, nt = len(self.blocks), len(self.text_refine_blocks)
        c = c.to(BF16)
        for j, blk in enumerate(self.text_refine_blocks):
            lin = blk.adaLN_modulation.lin
            mod = _ModFn.apply(c, lin.weight, lin)
            yt = _TextBlockFn.apply(yt, mod, blk.norm1.weight, blk, lens, T, (self, 1 + nb + (nt - 1 - j)), pack)
        # image tokens: Linear(Linear(patch)) + pos_embed
        h = _LinearFn.apply(x_tok, self.x_embedder.proj1.weight, self.x_embedder.proj1, False)
        h = _LinearFn.apply(h, self.x_embedder.proj2.weight, self.x_embedder.proj2, True)
        x = _AddRowsFn.apply(h, None, self.pos_embed.detach()[0], N, None)
        for i, blk in enumerate(self.blocks):
            lin = blk.adaLN_modulation.lin
            mod = _ModFn.apply(c, lin.weight, lin)
            x = _ImageBlockFn.apply(x, yt, mod, blk.norm1.weight, blk, lens, N, T, cos, sin, (self, nb - i), pack)
        x = _LayerNormFn.apply(x, 1e-6)
        return _LinearFn.apply(x, self.final_layer.linear.weight, self.final_layer.linear, True)

    def forward(self, x, t, y, return_layer=None, y_mask=None, y_pack=None):
        """x [B, C, H, W] -> predicted clean image [B, C, H, W] (fp32). Same call as the reference's forward, packed
        captions (y_pack) included; return_layer is not supported (the reference's ladder path does not use it)."""
        assert return_layer is None, "return_layer is not supported"
        B, Cin, H, W = x.shape
        tok = E.patchify(x.float(), self.patch_size)
        out = self.forward_tokens(tok, t, y, y_mask, y_pack)
        return _UnpatchifyFn.apply(out, (B, Cin, H, W), self.patch_size)
