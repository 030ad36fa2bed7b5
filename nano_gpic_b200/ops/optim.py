"""The optimizer's elementwise work as one launch each (csrc/optim.cu): the stacked Nesterov inputs of a shape's units,
`W <- W * decay + coef * O` over every Muon unit (the reference's Muon-add lever, baselines/PixelGen/src/optim/
muon_add.py:9-35, plus the weight decay that the reference applies with a separate _foreach_mul_), and AdamW over every
vector parameter (the reference's FusedAdamWEMA lever, baselines/PixelGen/src/utils/fused_adamw_ema.py:39-113); both
apply the EMA of the weights in the same pass when one is attached.

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


def stack_nesterov(grads, moms, beta, nesterov, update_momentum=False, dtype=torch.float32):
    """torch.stack([g.lerp(m, beta) if nesterov else m for g, m in zip(grads, moms)]) in `dtype` (fp32 or bf16), all
    of one shape. update_momentum: first m.lerp_(g, 1 - beta) for every pair (in the same pass on CUDA)."""
    if not all(_ok(g, torch.float32) and _ok(m, torch.float32) for g, m in zip(grads, moms)):
        if update_momentum:
            for g, m in zip(grads, moms):
                m.lerp_(g, 1 - beta)
        return torch.stack([g.lerp(m, beta) if nesterov else m for g, m in zip(grads, moms)]).to(dtype)
    out = torch.empty((len(grads),) + tuple(grads[0].shape), dtype=dtype, device=grads[0].device)
    rows = [[out[j].data_ptr(), g.data_ptr(), m.data_ptr(), g.numel()] for j, (g, m) in enumerate(zip(grads, moms))]
    ext().muon_gather(_table(rows, out.device), float(beta), bool(nesterov), grads[0].numel(),
                      float(1 - beta) if update_momentum else -1.0, dtype == torch.bfloat16)
    return out


def _f32_bits(x):
    return struct.unpack("<i", struct.pack("<f", float(x)))[0]


def apply_updates(items, decay, ema_w=0.0):
    """For each (param view fp32, update bf16 of the same shape, coef[, ema view fp32 or None]):
    param <- param * decay + coef * update, then ema <- lerp(ema, param, ema_w) where an EMA view is given."""
    def fits(it):
        return _ok(it[0], torch.float32) and _ok(it[1], torch.bfloat16) and (
            len(it) < 4 or it[3] is None or _ok(it[3], torch.float32))
    fast = [it for it in items if fits(it)]
    slow = [it for it in items if not fits(it)]
    if fast:
        with_ema = any(len(it) > 3 and it[3] is not None for it in fast)
        rows = [[it[0].data_ptr(), it[1].data_ptr(), it[0].numel(), _f32_bits(it[2])] +
                ([it[3].data_ptr() if len(it) > 3 and it[3] is not None else 0] if with_ema else []) for it in fast]
        ext().muon_apply(_table(rows, fast[0][0].device), float(decay), max(it[0].numel() for it in fast),
                         float(ema_w))
    for it in slow:
        p, o, c = it[:3]
        if decay != 1.0:
            p.mul_(decay)
        p.add_(o, alpha=c)
        if len(it) > 3 and it[3] is not None:
            it[3].lerp_(p, ema_w)


def adamw_update(params, grads, m1, m2, emas, lr, wd, b1, b2, eps, bc1, bc2, ema_w=0.0):
    """AdamW with decoupled weight decay on lists of fp32 tensors (torch.optim.AdamW's formula: p *= 1 - lr wd;
    m = lerp(m, g, 1 - b1); v = b2 v + (1 - b2) g^2; p -= (lr / bc1) m / (sqrt(v) / sqrt(bc2) + eps)), bias
    corrections bc1 = 1 - b1^t, bc2 = 1 - b2^t given; then ema = lerp(ema, p, ema_w) where emas[i] is not None.
    One launch for all of them on CUDA (csrc/optim.cu adamw_apply); the same arithmetic in PyTorch otherwise."""
    if not params:
        return
    emas = list(emas) if emas is not None else [None] * len(params)
    tensors = [t for group in (params, grads, m1, m2) for t in group] + [e for e in emas if e is not None]
    if all(_ok(t, torch.float32) for t in tensors):
        rows = [[p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), e.data_ptr() if e is not None else 0,
                 p.numel()] for p, g, m, v, e in zip(params, grads, m1, m2, emas)]
        ext().adamw_apply(_table(rows, params[0].device), [float(lr), float(wd), float(b1), float(b2), float(eps),
                                                           float(bc1), float(bc2), float(ema_w)],
                          max(p.numel() for p in params))
        return
    for p, g, m, v, e in zip(params, grads, m1, m2, emas):
        p.mul_(1 - lr * wd)
        m.lerp_(g, 1 - b1)
        v.mul_(b2).addcmul_(g, g, value=1 - b2)
        p.addcdiv_(m, v.sqrt().div_(bc2 ** 0.5).add_(eps), value=-lr / bc1)
        if e is not None:
            e.lerp_(p, ema_w)


def scale_(buf, coef):
    """buf *= coef in place, coef a one-element fp32 device tensor (the clip coefficient: no host read). One vectorized
    pass on CUDA (csrc/optim.cu scale_by) for contiguous, 16-byte aligned buffers of 4k values; PyTorch otherwise."""
    if (buf.is_cuda and buf.dtype == torch.float32 and buf.is_contiguous() and buf.numel() % 4 == 0
            and buf.data_ptr() % 16 == 0 and coef.is_cuda and coef.dtype == torch.float32 and coef.numel() == 1):
        ext().scale_by(buf, coef.reshape(1))
        return buf
    return buf.mul_(coef)


def ns_normalize(X, transpose=False):
    """Per matrix of X [n, a, b] (bf16): X / (||X||_F + 1e-7) with PyTorch's bf16 rounding, written as [n, b, a] when
    transpose (the Newton-Schulz input of tall matrices). One sum-of-squares pass and one scale pass on CUDA."""
    if not (X.is_cuda and X.dtype == torch.bfloat16 and X.dim() == 3 and X.is_contiguous() and X.shape[2] % 8 == 0):
        Y = X.mT if transpose else X
        return (Y / (Y.norm(dim=(-2, -1), keepdim=True) + 1e-7)).contiguous()
    n, a, b = X.shape
    out = torch.empty((n, b, a) if transpose else (n, a, b), dtype=X.dtype, device=X.device)
    ext().ns_normalize(X, bool(transpose), out)
    return out


def transpose_bf16(X):
    """[n, a, b] -> contiguous [n, b, a] (bf16, one tiled pass on CUDA)."""
    if not (X.is_cuda and X.dtype == torch.bfloat16 and X.dim() == 3 and X.is_contiguous()):
        return X.mT.contiguous()
    out = torch.empty((X.shape[0], X.shape[2], X.shape[1]), dtype=X.dtype, device=X.device)
    ext().transpose_bf16(X, out)
    return out
