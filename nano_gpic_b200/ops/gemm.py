"""bf16 GEMMs on the tcgen05 kernel (csrc/gemm.cu), with the epilogues the model fuses into them.

Every function takes 2-D row-major tensors (last stride 1) and returns new tensors unless an `out` is given. On CPU
tensors they compute the same formulas with PyTorch (fp32 math, bf16 rounding where the kernel rounds), which is
what the CPU tests and the CPU plumbing path use.

Reference sites: every nn.Linear under bf16 autocast in baselines/PixelGen/src/models/transformer/JiT_T2I.py
(cuBLAS there), the SwiGLU of baselines/PixelGen/src/models/layers/swiglu.py:4-24 and the gated residual adds of
JiT_T2I.py:201-210.
"""
import torch

from .._ext import ext
from .elementwise import Segments, _rows

EPI_BF16, EPI_F32, EPI_AXPBY, EPI_GATED, EPI_SWIGLU, EPI_SWIGLU_BWD = range(6)


def _ld(t):
    assert t.stride(-1) == 1, "row-major operand expected"
    return t.stride(-2) if t.dim() >= 2 else t.shape[-1]


def _bs(t):
    return t.stride(0) if t.dim() == 3 else 0


def _call(A, a_mn, B, b_mn, out, epi, M, N, K, batch=1, b_rows=0, out2=None, bias=None, res=None, gate=None,
          rows_per_group=1, aux=None, half_n=0, alpha=1.0, beta=0.0, accumulate=False, seg=None):
    ext().gemm(A, a_mn, _ld(A), _bs(A), B, b_mn, _ld(B), _bs(B), b_rows, out, _ld(out), _bs(out), epi, M, N, K, batch,
               out2, _ld(out2) if out2 is not None else 0, bias, res, _ld(res) if res is not None else 0,
               _bs(res) if res is not None else 0, gate, _ld(gate) if gate is not None else 0, rows_per_group, aux,
               _ld(aux) if aux is not None else 0, half_n, float(alpha), float(beta), bool(accumulate), seg)
    return out


def _bf(t):
    return t.to(torch.bfloat16)


# ----------------------------------------------------------------------------------------------------------- linear
def linear(x, w, bias=None, out=None):
    """y = x @ w^T + bias: x [M, K] bf16, w [N, K] bf16, bias [N] fp32 or None -> [M, N] bf16."""
    M, K = x.shape
    N = w.shape[0]
    if not x.is_cuda:
        y = x.float() @ w.float().t()
        if bias is not None:
            y = y + bias.float()
        return y.to(torch.bfloat16) if out is None else out.copy_(y)
    out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16) if out is None else out
    return _call(x, False, w, False, out, EPI_BF16, M, N, K, bias=bias)


def linear_dgrad(dy, w, out=None):
    """dx = dy @ w: dy [M, N] bf16, w [N, K] bf16 -> [M, K] bf16."""
    M, N = dy.shape
    K = w.shape[1]
    if not dy.is_cuda:
        return (dy.float() @ w.float()).to(torch.bfloat16)
    out = torch.empty(M, K, device=dy.device, dtype=torch.bfloat16) if out is None else out
    # GEMM (M, K, N): A = dy K-major, B[k_out, n] = w[n, k_out]: w is [N, K] = [red, out] -> MN-major
    return _call(dy, False, w, True, out, EPI_BF16, M, K, N)


def linear_wgrad(dy, x, out=None, accumulate=False):
    """dw (+)= dy^T @ x in fp32: dy [M, N] bf16, x [M, K] bf16 -> [N, K] fp32."""
    M, N = dy.shape
    K = x.shape[1]
    if not dy.is_cuda:
        g = dy.float().t() @ x.float()
        if out is None:
            return g
        return out.add_(g) if accumulate else out.copy_(g)
    if out is None:
        out = torch.empty(N, K, device=dy.device, dtype=torch.float32)
        accumulate = False
    # GEMM (N, K, M): A[n, m] = dy[m, n] -> dy is [red, rows] = MN-major; B[k, m] = x[m, k] -> MN-major
    return _call(dy, True, x, True, out, EPI_F32, N, K, M, accumulate=accumulate)


def linear_wgrad_bf16(dy, x):
    """dw = dy^T @ x rounded to bf16 (for bf16 gradient buckets)."""
    M, N = dy.shape
    K = x.shape[1]
    if not dy.is_cuda:
        return (dy.float().t() @ x.float()).to(torch.bfloat16)
    out = torch.empty(N, K, device=dy.device, dtype=torch.bfloat16)
    return _call(dy, True, x, True, out, EPI_BF16, N, K, M)


# ------------------------------------------------------------------------------------------------- fused epilogues
def linear_gated_residual(x, w, bias, res, gate, rows_per_group):
    """y = bf16(x @ w^T + bias); out = bf16(res + gate[row // rows_per_group] * y). Returns (out, y).
    gate: [G, N] bf16 with a row stride of its own (e.g. a column slice of the adaLN output). rows_per_group may be a
    Segments (packed rows: the gate row of each row from its segment table)."""
    M, K = x.shape
    N = w.shape[0]
    seg = rows_per_group if isinstance(rows_per_group, Segments) else None
    if not x.is_cuda:
        y = x.float() @ w.float().t()
        if bias is not None:
            y = y + bias.float()
        y = y.to(torch.bfloat16)
        g = _rows(rows_per_group, gate.float(), M)
        return (res.float() + g * y.float()).to(torch.bfloat16), y
    out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    y = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    _call(x, False, w, False, out, EPI_GATED, M, N, K, out2=y, bias=bias, res=res, gate=gate,
          rows_per_group=1 if seg is not None else rows_per_group, seg=seg.seg if seg is not None else None)
    return out, y


def swiglu_linear(x, w12):
    """pre = bf16(x @ w12^T) [M, 2H]; act = bf16(silu(pre[:, :H]) * pre[:, H:]) [M, H]. Returns (act, pre)."""
    M, K = x.shape
    H2 = w12.shape[0]
    H = H2 // 2
    if not x.is_cuda:
        pre = (x.float() @ w12.float().t()).to(torch.bfloat16)
        x1, x2 = pre.float().chunk(2, dim=-1)
        act = (torch.nn.functional.silu(x1).to(torch.bfloat16).float() * x2).to(torch.bfloat16)
        return act, pre
    act = torch.empty(M, H, device=x.device, dtype=torch.bfloat16)
    pre = torch.empty(M, H2, device=x.device, dtype=torch.bfloat16)
    _call(x, False, w12, False, act, EPI_SWIGLU, M, H2, K, b_rows=H2, out2=pre, half_n=H)
    return act, pre


def swiglu_dgrad(dy, w3, pre):
    """d(act) = dy @ w3, then the SwiGLU backward against the saved pre-activation: returns d(pre) [M, 2H] bf16."""
    M, N = dy.shape
    H = w3.shape[1]
    if not dy.is_cuda:
        da = dy.float() @ w3.float()
        x1, x2 = pre.float().chunk(2, dim=-1)
        s = torch.sigmoid(x1)
        d1 = da * x2 * (s * (1 + x1 * (1 - s)))
        d2 = da * x1 * s
        return torch.cat([d1, d2], dim=-1).to(torch.bfloat16)
    out = torch.empty(M, 2 * H, device=dy.device, dtype=torch.bfloat16)
    _call(dy, False, w3, True, out, EPI_SWIGLU_BWD, M, H, N, aux=pre, half_n=H)
    return out


def bmm_axpby(A, B, b_mn, alpha=1.0, beta=0.0, C=None, out=None):
    """Batched out = alpha * A @ op(B) + beta * C in bf16 (fp32 accumulate).
    A [b, M, K]; B [b, N, K] (b_mn False: out = A B^T) or [b, K, N] (b_mn True: out = A B); C [b, M, N] or None."""
    if A.dim() == 2:
        A, B = A.unsqueeze(0), B.unsqueeze(0)
        C = C.unsqueeze(0) if C is not None else None
        squeeze = True
    else:
        squeeze = False
    bt, M, K = A.shape
    N = B.shape[2] if b_mn else B.shape[1]
    if not A.is_cuda:
        Bm = B.float() if b_mn else B.float().transpose(1, 2)
        r = alpha * (A.float() @ Bm)
        if C is not None and beta != 0.0:
            r = r + beta * C.float()
        r = r.to(torch.bfloat16)
        return r[0] if squeeze else r
    if out is None:
        out = torch.empty(bt, M, N, device=A.device, dtype=torch.bfloat16)
    _call(A, False, B, b_mn, out, EPI_AXPBY, M, N, K, batch=bt, res=C if beta != 0.0 else None, alpha=alpha,
          beta=beta if C is not None else 0.0)
    return out[0] if squeeze else out
