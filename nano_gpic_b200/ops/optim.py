"""Muon's per-unit elementwise work as one launch each (csrc/optim.cu): the stacked Nesterov inputs of a shape's units
and `W <- W * decay + coef * O` over every unit (the reference's Muon-add lever, baselines/PixelGen/src/optim/
muon_add.py:9-35, plus the weight decay that the reference applies with a separate _foreach_mul_).

The kernels read device pointer tables (int64 rows) built here each call. Operands that are not contiguous, not
16-byte aligned, or whose size is not a multiple of 4 take the PyTorch path, as do CPU tensors.
"""
import struct

import torch

from .._ext import ext


def _table(rows, device):
    t = torch.tensor(rows, dtype=torch.int64).pin_memory()
    return t.to(device, non_blocking=True)


def _ok(t, dtype):
    return t.is_cuda and t.dtype == dtype and t.is_contiguous() and t.numel() % 4 == 0 and t.data_ptr() % 16 == 0


def stack_nesterov(grads, moms, beta, nesterov):
    """torch.stack([g.lerp(m, beta) if nesterov else m for g, m in zip(grads, moms)]) (fp32, all of one shape)."""
    if not all(_ok(g, torch.float32) and _ok(m, torch.float32) for g, m in zip(grads, moms)):
        return torch.stack([g.lerp(m, beta) if nesterov else m for g, m in zip(grads, moms)])
    out = torch.empty((len(grads),) + tuple(grads[0].shape), dtype=torch.float32, device=grads[0].device)
    rows = [[out[j].data_ptr(), g.data_ptr(), m.data_ptr(), g.numel()] for j, (g, m) in enumerate(zip(grads, moms))]
    ext().muon_gather(_table(rows, out.device), float(beta), bool(nesterov), grads[0].numel())
    return out


def _f32_bits(x):
    return struct.unpack("<i", struct.pack("<f", float(x)))[0]


def apply_updates(items, decay):
    """For each (param view fp32, update bf16 of the same shape, coef): param <- param * decay + coef * update."""
    fast = [it for it in items if _ok(it[0], torch.float32) and _ok(it[1], torch.bfloat16)]
    slow = [it for it in items if not (_ok(it[0], torch.float32) and _ok(it[1], torch.bfloat16))]
    if fast:
        rows = [[p.data_ptr(), o.data_ptr(), p.numel(), _f32_bits(c)] for p, o, c in fast]
        ext().muon_apply(_table(rows, fast[0][0].device), float(decay), max(p.numel() for p, _, _ in fast))
    for p, o, c in slow:
        if decay != 1.0:
            p.mul_(decay)
        p.add_(o, alpha=c)
