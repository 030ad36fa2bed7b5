"""tcgen05 GEMM (csrc/gemm.cu) against fp32 PyTorch references, every operand layout and epilogue."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _r(*s, scale=1.0):
    return (torch.randn(*s, device="cuda") * scale).to(torch.bfloat16)


def _close(a, b, rtol=2e-2, atol=2e-2):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= atol + rtol * ref, f"max err {err} vs ref max {ref}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 520, 200), (1024, 3072, 1024), (77, 8, 40)])
def test_linear_fwd(M, N, K):
    from nano_gpic_b200.ops import gemm
    x, w = _r(M, K), _r(N, K, scale=0.05)
    b = torch.randn(N, device="cuda")
    y = gemm.linear(x, w, b)
    _close(y, x.float() @ w.float().t() + b)
    torch.cuda.synchronize()
    from nano_gpic_b200.ops import status
    assert status.read() == 0


@pytest.mark.parametrize("M,N,K", [(256, 512, 128), (300, 136, 200), (2048, 1024, 4096)])
def test_linear_dgrad(M, N, K):
    from nano_gpic_b200.ops import gemm
    dy, w = _r(M, N), _r(N, K, scale=0.05)
    _close(gemm.linear_dgrad(dy, w), dy.float() @ w.float())


@pytest.mark.parametrize("M,N,K", [(256, 512, 128), (300, 136, 200), (4096, 1024, 1024)])
def test_linear_wgrad(M, N, K):
    from nano_gpic_b200.ops import gemm
    dy, x = _r(M, N, scale=0.1), _r(M, K)
    ref = dy.float().t() @ x.float()
    out = gemm.linear_wgrad(dy, x)
    _close(out, ref, rtol=1e-2, atol=1e-2)
    gemm.linear_wgrad(dy, x, out=out, accumulate=True)
    _close(out, 2 * ref, rtol=1e-2, atol=2e-2)


def test_gated_residual():
    from nano_gpic_b200.ops import gemm
    B, L, C = 4, 256, 512
    x, w = _r(B * L, C), _r(C, C, scale=0.05)
    bias = torch.randn(C, device="cuda")
    res = _r(B * L, C)
    mod = _r(B, 6 * C)
    gate = mod[:, 2 * C:3 * C]
    out, y = gemm.linear_gated_residual(x, w, bias, res, gate, L)
    yr = (x.float() @ w.float().t() + bias).bfloat16()
    _close(y, yr)
    ref = res.float() + gate.float().repeat_interleave(L, 0) * yr.float()
    _close(out, ref)


def test_swiglu_fwd_bwd():
    from nano_gpic_b200.ops import gemm
    M, C, H = 512, 256, 1024
    x, w12, w3 = _r(M, C), _r(2 * H, C, scale=0.05), _r(C, H, scale=0.05)
    act, pre = gemm.swiglu_linear(x, w12)
    pr = (x.float() @ w12.float().t())
    _close(pre, pr)
    x1, x2 = pre.float().chunk(2, -1)
    _close(act, torch.nn.functional.silu(x1) * x2)
    dy = _r(M, C)
    dpre = gemm.swiglu_dgrad(dy, w3, pre)
    x1r = x1.clone().requires_grad_(True)
    x2r = x2.clone().requires_grad_(True)
    h = torch.nn.functional.silu(x1r) * x2r
    (h @ w3.float().t()).backward(dy.float())
    _close(dpre, torch.cat([x1r.grad, x2r.grad], -1))


@pytest.mark.parametrize("b_mn", [False, True])
def test_bmm_axpby(b_mn):
    from nano_gpic_b200.ops import gemm
    bt, M, N, K = 3, 256, 256, 384
    A = _r(bt, M, K)
    B = _r(bt, K, N) if b_mn else _r(bt, N, K)
    C = _r(bt, M, N)
    out = gemm.bmm_axpby(A, B, b_mn, alpha=0.5, beta=-1.5, C=C)
    Bm = B.float() if b_mn else B.float().transpose(1, 2)
    _close(out, 0.5 * (A.float() @ Bm) - 1.5 * C.float())


@pytest.mark.parametrize("pair", [True, False])
def test_pair_and_single_cta_agree(pair):
    """The CTA-pair (cta_group::2) tiles and the single-CTA tiles give the same results on every operand layout."""
    from nano_gpic_b200 import _ext
    from nano_gpic_b200.ops import gemm as G, status
    torch.manual_seed(5)
    x, w, dy = _r(600, 512), _r(768, 512, scale=0.05), _r(600, 768)
    try:
        _ext.ext().gemm_set_pair(1 if pair else 0)
        y = G.linear(x, w)
        dx = G.linear_dgrad(dy, w)
        dw = G.linear_wgrad(dy, x)
    finally:
        _ext.ext().gemm_set_pair(1)
    ref_y = (x.float() @ w.float().t())
    ref_dx = (dy.float() @ w.float())
    ref_dw = (dy.float().t() @ x.float())
    for a, b, name in ((y, ref_y, "fwd"), (dx, ref_dx, "dgrad"), (dw, ref_dw, "wgrad")):
        err = (a.float() - b).abs().max().item()
        assert err <= 2e-2 * b.abs().max().item() + 1e-2, (name, pair, err)
    assert status.read() == 0
