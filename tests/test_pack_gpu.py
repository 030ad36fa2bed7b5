"""Packed captions on the GPU kernels (segment tables in the RMSNorm+modulate forward/backward, the gated GEMM
epilogue and the gate backward; row gathers to and from the padded attention layout) against the padded, masked run
of the same model, and the segment-aware kernels against their PyTorch forms."""
import pytest
import torch

from test_pack_cpu import TINY, _inputs

pytestmark = pytest.mark.gpu


def _model_cuda(seed=0):
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    from nano_gpic_b200.parallel.flat import FlatParams
    torch.manual_seed(seed)
    m = JiT_T2I(**TINY)
    with torch.no_grad():
        for p in m.parameters():
            if p.requires_grad:
                p.copy_(torch.randn_like(p) * (0.2 if p.ndim == 2 else 0.05) + (1.0 if p.ndim == 1 and p.numel() in
                                                                                   (64, 128) else 0.0))
    m = m.cuda()
    FlatParams(m, device="cuda")
    return m


def test_segment_kernels_match_torch():
    from nano_gpic_b200.ops import elementwise as E
    from nano_gpic_b200.ops import gemm as G
    from nano_gpic_b200.ops import norm as NR
    torch.manual_seed(0)
    lens = [70, 1, 129, 0, 64]
    B, C = len(lens), 256
    s_real = sum(lens)
    S = s_real + 37
    seg = torch.cat([torch.full((n,), b) for b, n in enumerate(lens)] + [torch.full((S - s_real,), B)])
    cu = torch.tensor([0] + torch.cumsum(torch.tensor(lens), 0).tolist())
    segs = {}
    for dev in ("cpu", "cuda"):
        segs[dev] = E.Segments(seg.int().to(dev), cu.int().to(dev), max(lens))
    x = torch.randn(S, C).bfloat16()
    mod = torch.cat([torch.randn(B, 6 * C).bfloat16() * 0.3, torch.zeros(1, 6 * C).bfloat16()])
    w = torch.randn(C) * 0.1 + 1
    dh = torch.randn(S, C).bfloat16()
    dres = torch.randn(S, C).bfloat16()
    W = (torch.randn(C, C) * 0.05).bfloat16()
    res = {}
    for dev in ("cpu", "cuda"):
        sg = segs[dev]
        xd, md, wd = x.to(dev), mod.to(dev), w.to(dev)
        h, r = NR.rms_mod_fwd(xd, wd, md[:, 0:C], md[:, C:2 * C], sg)
        dmod = torch.zeros(B + 1, 6 * C, device=dev)
        dw = torch.zeros(C, device=dev)
        dx = NR.rms_mod_bwd(dh.to(dev), xd, r, wd, md[:, C:2 * C], sg, dres=dres.to(dev), dw_acc=dw,
                            dshift=dmod[:, 0:C], dscale=dmod[:, C:2 * C])
        out, y = G.linear_gated_residual(h, W.to(dev), None, xd, md[:, 2 * C:3 * C], sg)
        db = torch.zeros(C, device=dev)
        dy = E.gate_bwd(dh.to(dev), y, md[:, 2 * C:3 * C], sg, dgate=dmod[:, 2 * C:3 * C], dbias=db)
        res[dev] = [t.float().cpu() for t in (h, r, dx, dmod[:B], dw, out, y, dy, db)]
    names = ["h", "rstd", "dx", "dmod", "dw", "out", "y", "dy", "dbias"]
    for n, a, b in zip(names, res["cuda"], res["cpu"]):
        torch.testing.assert_close(a, b, rtol=2e-2, atol=2e-2, msg=n)
    assert not res["cuda"][2][s_real:].any() and not res["cuda"][7][s_real:].any()  # dummy rows: zero gradients


def test_packed_matches_masked_on_gpu():
    from nano_gpic_b200.parallel.rebalance import pack_captions
    lens, T = [5, 16, 1, 9], 16
    x, t, y, mask = (v.cuda() for v in _inputs(lens, T))
    w = torch.randn(4, 3, 64, 64, device="cuda")
    outs, grads = [], []
    for packed in (False, True):
        m = _model_cuda()
        if packed:
            yp, pk = pack_captions(y, mask, lens=lens, bucket=128)
            out = m(x, t, yp, y_pack=pk)
        else:
            out = m(x, t, y, y_mask=mask)
        (out.float() * w).sum().backward()
        outs.append(out.float().detach())
        grads.append({n: p.grad.clone() for n, p in m.named_parameters() if p.requires_grad})
    torch.testing.assert_close(outs[1], outs[0], rtol=2e-2, atol=5e-2)
    bad = []
    for n, g0 in grads[0].items():
        e = (grads[1][n] - g0).norm().item() / (g0.norm().item() + 1e-8)
        if e > 2e-2:
            bad.append((n, round(e, 4)))
    assert not bad, bad
