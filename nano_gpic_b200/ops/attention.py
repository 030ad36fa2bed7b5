"""Masked multi-head attention (head dim 64) over up to two key/value sources, forward and backward.

Sample b's queries (Lq rows) attend to n0[b] keys of source 0 followed by n1[b] keys of source 1:
    image blocks   source 0 = the 256 image keys (RoPE'd), source 1 = the caption keys, n1[b] = caption length
    text blocks    source 0 = the caption keys, n0[b] = caption length, no source 1
which is the reference's joint attention with a key-padding mask (SDPA, or FA3 with seqused_k;
baselines/PixelGen/src/models/transformer/JiT_T2I.py:114-187, 212-265, baselines/PixelGen/src/models/layers/fa3_op.py)
without materialising the concatenated keys. softmax scale = 1/8. Forward also returns the log-sum-exp (natural log)
per (sample, head, query) for the backward. Gradients of padded keys are zero.

All tensors are token-major 2-D views [rows, H*64] with their own row strides (e.g. the v part of the fused qkv
projection), last stride 1.
"""
import torch

from .._ext import ext

HEAD = 64
_VERSIONS = {"tc": 3, "tc2": 2, "tc1": 1}  # kernel versions of csrc/attn_tc.cu


def _lens(n, B, device):
    if isinstance(n, int):
        return torch.full((B,), n, dtype=torch.int32, device=device)
    return n.to(device=device, dtype=torch.int32)


def _keys_cpu(k0, v0, L0, n0, k1, v1, L1, n1, B, H):
    ks, vs, masks = [], [], []
    for b in range(B):
        kb = [k0[b * L0:(b + 1) * L0]]
        vb = [v0[b * L0:(b + 1) * L0]]
        m = [torch.arange(L0) < int(n0[b])]
        if k1 is not None:
            kb.append(k1[b * L1:(b + 1) * L1])
            vb.append(v1[b * L1:(b + 1) * L1])
            m.append(torch.arange(L1) < int(n1[b]))
        ks.append(torch.cat(kb).float().view(-1, H, HEAD).transpose(0, 1))
        vs.append(torch.cat(vb).float().view(-1, H, HEAD).transpose(0, 1))
        masks.append(torch.cat(m))
    return torch.stack(ks), torch.stack(vs), torch.stack(masks)


def attn_fwd(q, Lq, k0, v0, L0, n0, k1=None, v1=None, L1=0, n1=None, scale=0.125, impl="tc"):
    """q [B*Lq, H*64]; k0/v0 [B*L0, H*64]; k1/v1 [B*L1, H*64] or None; n0/n1: int or int32 [B] valid-key counts.
    Returns (o [B*Lq, H*64] bf16, lse [B, H, Lq] fp32). On CUDA the forward runs on tcgen05/TMEM
    (csrc/attn_tc.cu; impl="tc", the default: version 3, a persistent kernel with two query tiles per CTA, S released
    as soon as it is in registers, P double-buffered, O rescaled only when a row maximum grows by more than 2^8;
    impl="tc2": version 2, the same two-tile ping-pong without those three; impl="tc1": one 128-query tile per CTA);
    impl="mma" selects the warp-level mma.sync kernel (csrc/attention.cu), kept as a test oracle."""
    rows, C = q.shape
    B, H = rows // Lq, C // HEAD
    n0 = _lens(n0, B, q.device)
    n1 = _lens(n1 if n1 is not None else 0, B, q.device)
    if not q.is_cuda:
        K, V, mask = _keys_cpu(k0, v0, L0, n0, k1, v1, L1, n1, B, H)
        Q = q.float().view(B, Lq, H, HEAD).transpose(1, 2)
        s = (Q @ K.transpose(-1, -2)) * scale
        s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
        lse = torch.logsumexp(s, -1)
        p = torch.exp(s - lse[..., None])
        o = (p @ V).transpose(1, 2).reshape(rows, C)
        return o.to(torch.bfloat16), lse
    o = torch.empty(rows, C, device=q.device, dtype=torch.bfloat16)
    lse = torch.empty(B, H, Lq, device=q.device, dtype=torch.float32)
    if impl in _VERSIONS:
        ext().attn_fwd_tc(q, k0, v0, k1, v1, n0, n1, o, lse, Lq, L0, L1, scale, _VERSIONS[impl])
    else:
        ext().attn_fwd(q, k0, v0, k1, v1, n0, n1, o, lse, Lq, L0, L1, scale)
    return o, lse


def attn_bwd(do, q, Lq, k0, v0, L0, n0, o, lse, k1=None, v1=None, L1=0, n1=None, scale=0.125,
             dq=None, dk0=None, dv0=None, dk1=None, dv1=None, impl="tc"):
    """Gradients of attn_fwd. dq/dk*/dv* may be given as (strided) views to write into; missing ones are allocated.
    Returns (dq, dk0, dv0, dk1, dv1). On CUDA the backward runs on tcgen05/TMEM (csrc/attn_tc.cu; impl="tc", the
    default: version 3, a persistent CTA per (sample, head) with dQ of its (at most two) query tiles accumulated in
    TMEM over the key tiles and dK/dV per key tile over the query tiles; longer query sets take version 2;
    impl="tc2": version 2, a persistent CTA per key tile whose dQ partials are summed by TMA reduce-adds; impl="tc1":
    one CTA per key tile); impl="mma" selects the mma.sync kernels."""
    rows, C = q.shape
    B, H = rows // Lq, C // HEAD
    n0 = _lens(n0, B, q.device)
    n1 = _lens(n1 if n1 is not None else 0, B, q.device)
    if not q.is_cuda:
        with torch.enable_grad():
            K, V, mask = _keys_cpu(k0, v0, L0, n0, k1, v1, L1, n1, B, H)
            K.requires_grad_(True)
            V.requires_grad_(True)
            Q = q.float().view(B, Lq, H, HEAD).transpose(1, 2).clone().requires_grad_(True)
            s = (Q @ K.transpose(-1, -2)) * scale
            s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
            p = torch.softmax(s, -1)
            out = (p @ V).transpose(1, 2).reshape(rows, C)
            out.backward(do.float())
        gq = Q.grad.transpose(1, 2).reshape(rows, C)
        gk, gv = K.grad.transpose(1, 2), V.grad.transpose(1, 2)  # [B, L0+L1, H, 64]
        gk = gk * mask[..., None, None]
        gv = gv * mask[..., None, None]
        res = [gq]
        outs = [dq]
        res += [gk[:, :L0].reshape(B * L0, C), gv[:, :L0].reshape(B * L0, C)]
        outs += [dk0, dv0]
        if k1 is not None:
            res += [gk[:, L0:].reshape(B * L1, C), gv[:, L0:].reshape(B * L1, C)]
            outs += [dk1, dv1]
        final = []
        for r, dst in zip(res, outs):
            r = r.to(torch.bfloat16)
            if dst is not None:
                dst.copy_(r)
                final.append(dst)
            else:
                final.append(r)
        while len(final) < 5:
            final.append(None)
        return tuple(final)

    def alloc(t, n):
        return t if t is not None else torch.empty(n, C, device=q.device, dtype=torch.bfloat16)
    dq = alloc(dq, rows)
    dk0 = alloc(dk0, B * L0)
    dv0 = alloc(dv0, B * L0)
    if k1 is not None:
        dk1 = alloc(dk1, B * L1)
        dv1 = alloc(dv1, B * L1)
    if impl in _VERSIONS:
        ext().attn_bwd_tc(do, q, k0, v0, k1, v1, n0, n1, o, lse, dq, dk0, dv0, dk1, dv1, Lq, L0, L1, scale,
                          _VERSIONS[impl])
    else:
        ext().attn_bwd(do, q, k0, v0, k1, v1, n0, n1, o, lse, dq, dk0, dv0, dk1, dv1, Lq, L0, L1, scale)
    return dq, dk0, dv0, dk1, dv1
