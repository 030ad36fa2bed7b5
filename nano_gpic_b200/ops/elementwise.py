"""Memory-bound ops around the GEMMs (csrc/elementwise.cu), each with its PyTorch path for CPU tensors.

Reference sites: gated residual adds (baselines/PixelGen/src/models/transformer/JiT_T2I.py:201-210), the
flow-matching objective (baselines/PixelGen/src/diffusion/flow_matching/training_JiT.py:36-64), patchify/unpatchify
(JiT_T2I.py:42-52, 463-476) and the position-table adds (JiT_T2I.py:508, 513-514).
"""
import torch

from .._ext import ext


class Segments:
    """Packed rows grouped by sample (the reference's packed captions, JiT_T2I.py:54-65): row r takes the modulation
    row seg[r] ([S] int32; rows after the last sample point at a zero row); sample g owns rows [cu[g], cu[g + 1])
    ([G + 1] int32), at most max_rows of them. Ops that take `rows_per_group` accept a Segments in its place: forward
    kernels read seg, backward reductions read cu, and rows after cu[G] get zero gradients."""

    def __init__(self, seg, cu, max_rows):
        self.seg, self.cu, self.max_rows = seg, cu, int(max_rows)
        self.groups = cu.numel() - 1

    def expand(self, t):
        """t [G (+ 1), C] -> [S, C]: each row's group row (PyTorch; the CPU paths)."""
        return t.index_select(0, self.seg.long())

    def sum_rows(self, v):
        """[S, C] -> [G, C]: per-group sums of the rows each group owns (PyTorch; the CPU paths)."""
        owned = self.seg.long() < self.groups
        out = torch.zeros(self.groups, v.shape[1], dtype=v.dtype, device=v.device)
        return out.index_add_(0, self.seg.long()[owned], v[owned])

    def owned(self, M, device):
        """[M] bool: rows that belong to a group."""
        return self.seg.long().to(device) < self.groups


def _rows(rows_per_group, t, M):
    """t [G, C] expanded to one row per token for the PyTorch paths."""
    if isinstance(rows_per_group, Segments):
        return rows_per_group.expand(t)
    return t.repeat_interleave(rows_per_group, 0)[:M]


def gate_bwd(dout, y, gate, rows_per_group, dgate=None, dbias=None):
    """Backward of out = res + gate[row // rows_per_group] * y (res's gradient is dout itself); rows_per_group may be
    a Segments (packed rows).
    Returns dy = bf16(gate * dout); writes d_gate [G, C] into `dgate` (fp32 view) and adds d_bias (the column sums of
    the rounded dy) into `dbias` [C] fp32 when given."""
    M, C = dout.shape
    seg = rows_per_group if isinstance(rows_per_group, Segments) else None
    if not dout.is_cuda:
        g = _rows(rows_per_group, gate.float(), M)
        dy = (g * dout.float()).to(torch.bfloat16)
        if seg is not None:
            dy = dy * seg.owned(M, dy.device)[:, None].to(dy.dtype)
        if dgate is not None:
            prod = dout.float() * y.float()
            if seg is not None:
                dgate[:seg.groups].copy_(seg.sum_rows(prod))
            else:
                dgate.copy_(prod.view(gate.shape[0], rows_per_group, C).sum(1))
        if dbias is not None:
            dbias.add_(dy.float().sum(0))
        return dy
    if seg is not None:
        dy = torch.zeros_like(dout)  # rows of no sample keep a zero gradient
        ext().gate_bwd(dout, y, gate, dy, dgate, dbias, 1, seg.cu, seg.max_rows)
        return dy
    dy = torch.empty_like(dout)
    ext().gate_bwd(dout, y, gate, dy, dgate, dbias, rows_per_group, None, 0)
    return dy


def gather_rows(src, idx, out=None):
    """out[r] = src[idx[r]] for bf16 rows (zeros where idx[r] < 0): src [R, C] (row stride free), idx [M] int32 ->
    [M, C]. Moves caption rows between the packed layout and the padded [B, Tp] layout."""
    M, C = idx.numel(), src.shape[1]
    if out is None:
        out = torch.empty(M, C, dtype=src.dtype, device=src.device)
    if not src.is_cuda:
        i = idx.long()
        vals = src.index_select(0, i.clamp(min=0))
        out.copy_(vals * (i >= 0)[:, None].to(vals.dtype))
        return out
    ext().gather_rows(src, idx, out)
    return out


def _patch_index(B, Cin, H, W, p, device):
    gh, gw = H // p, W // p
    return torch.arange(B * Cin * H * W, device=device).view(B, Cin, gh, p, gw, p).permute(0, 2, 4, 1, 3, 5).reshape(
        B * gh * gw, Cin * p * p)


def patchify(img, p):
    """[B, C, H, W] -> bf16 tokens [B*(H/p)*(W/p), C*p*p], vector order (c, py, px) as F.unfold."""
    B, Cin, H, W = img.shape
    if not img.is_cuda:
        return img.reshape(-1)[_patch_index(B, Cin, H, W, p, img.device)].to(torch.bfloat16)
    tok = torch.empty(B * (H // p) * (W // p), Cin * p * p, device=img.device, dtype=torch.bfloat16)
    ext().patchify(img.contiguous(), tok, p)
    return tok


def unpatchify(tok, B, Cin, H, W, p, dtype=torch.float32):
    """Inverse of patchify (F.fold of non-overlapping patches)."""
    if not tok.is_cuda:
        out = torch.empty(B * Cin * H * W, dtype=dtype)
        out[_patch_index(B, Cin, H, W, p, tok.device).reshape(-1)] = tok.reshape(-1).to(dtype)
        return out.view(B, Cin, H, W)
    img = torch.empty(B, Cin, H, W, device=tok.device, dtype=dtype)
    ext().unpatchify(tok.contiguous(), img, p)
    return img


def fm_prep(x, noise, t, p):
    """x_t = t x + (1 - t) noise (per-sample t), patchified to bf16 tokens."""
    if not x.is_cuda:
        tt = t.view(-1, 1, 1, 1).float()
        return patchify(tt * x + noise * (1 - tt), p)
    B, Cin, H, W = x.shape
    tok = torch.empty(B * (H // p) * (W // p), Cin * p * p, device=x.device, dtype=torch.bfloat16)
    ext().fm_prep(x.float().contiguous(), noise.float().contiguous(), t.float().contiguous(), tok, p)
    return tok


def fm_loss(pred_tok, x, noise, t, p, t_eps=0.05, grad_scale=None, need_grad=True):
    """Per-sample mean of (out - v)^2 over C,H,W with out = (pred - x_t)/d, v = (x - x_t)/d, d = max(1 - t, t_eps).
    Returns (loss_per_sample [B] fp32, d(grad_scale * sum of squares)/d pred as bf16 tokens or None).
    grad_scale defaults to 1 / numel(x), the gradient of the batch mean."""
    B = x.shape[0]
    if grad_scale is None:
        grad_scale = 1.0 / x.numel()
    if not x.is_cuda:
        tt = t.view(-1, 1, 1, 1).float()
        xt = tt * x + noise * (1 - tt)
        den = (1 - tt).clamp_min(t_eps)
        pred = unpatchify(pred_tok, *x.shape, p)
        d = (pred - xt) / den - (x - xt) / den
        per = d.pow(2).mean(dim=(1, 2, 3))
        g = patchify(grad_scale * 2 * d / den, p) if need_grad else None
        return per, g
    per = torch.empty(B, device=x.device, dtype=torch.float32)
    g = torch.empty_like(pred_tok) if need_grad else None
    ext().fm_loss(pred_tok.contiguous(), x.float().contiguous(), noise.float().contiguous(), t.float().contiguous(), g,
                  per, p, t_eps, grad_scale)
    return per, g


def colsum(src, out, accumulate=True):
    """out (+)= column sums of src [rows, C] (fp32 or bf16), deterministic, fp32 accumulation."""
    if not src.is_cuda:
        t = src.float().sum(0)
        return out.add_(t) if accumulate else out.copy_(t)
    ext().colsum(src, out, accumulate)
    return out


def add_rows(a, table, period):
    """bf16(a[row] + table[row % period]): a [rows, C] bf16, table [period, C] fp32 or bf16."""
    if not a.is_cuda:
        rows = a.shape[0]
        idx = torch.arange(rows) % period
        return (a.float() + table.float()[idx]).to(torch.bfloat16)
    out = torch.empty_like(a)
    ext().add_rows(a, table.contiguous(), out, period)
    return out
