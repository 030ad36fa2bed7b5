"""Table-driven Muon kernels (csrc/optim.cu) against the PyTorch formulas they replace, and one MuonAdamW step with them
against the same step on the PyTorch path."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_stack_nesterov_and_apply_match_torch():
    from nano_gpic_b200.ops import optim as OPT
    torch.manual_seed(0)
    P = [torch.randn(3 * 256, 128, device="cuda") for _ in range(3)]
    G = [torch.randn_like(p) for p in P]
    M = [torch.randn_like(p) for p in P]
    gs = [g[256:512] for g in G]
    ms = [m[256:512] for m in M]
    for nesterov in (True, False):
        got = OPT.stack_nesterov(gs, ms, 0.95, nesterov)
        ref = torch.stack([g.lerp(m, 0.95) if nesterov else m for g, m in zip(gs, ms)])
        torch.testing.assert_close(got, ref, rtol=1e-6, atol=1e-6)
    O = [torch.randn(256, 128, device="cuda").to(torch.bfloat16) for _ in range(3)]
    ref = [p.clone() for p in P]
    for r, o, c in zip(ref, O, (-0.1, 0.2, -0.3)):
        r[:256].mul_(0.99).add_(o, alpha=c)
        r[256:].mul_(0.99)
    items = [(p[:256], o, c) for p, o, c in zip(P, O, (-0.1, 0.2, -0.3))]
    items += [(p[256:512], torch.zeros_like(o), 0.0) for p, o in zip(P, O)]
    items += [(p[512:], torch.zeros_like(o), 0.0) for p, o in zip(P, O)]
    OPT.apply_updates(items, 0.99)
    for p, r in zip(P, ref):
        torch.testing.assert_close(p, r, rtol=1e-6, atol=1e-6)


def test_muon_step_fused_matches_torch_path(monkeypatch):
    from nano_gpic_b200.ops import optim as OPT
    from nano_gpic_b200.optim.muon import MuonAdamW

    def run(fused):
        torch.manual_seed(1)
        ws = [torch.nn.Parameter(torch.randn(3 * 128, 256, device="cuda") * 0.02),
              torch.nn.Parameter(torch.randn(512, 128, device="cuda") * 0.02),
              torch.nn.Parameter(torch.randn(256, device="cuda"))]
        ws[0]._muon_parts, ws[1]._muon_parts = 3, 1
        opt = MuonAdamW(ws, lr=1e-3, weight_decay=0.0, muon_lr=2e-2, muon_weight_decay=0.1, split=True,
                        ns_dtype="bfloat16")
        if not fused:
            monkeypatch.setattr(OPT, "_ok", lambda t, dtype: False)
        for step in range(2):
            for w in ws:
                w.grad = torch.randn_like(w)
            opt.step()
        monkeypatch.undo()
        return [w.detach().clone() for w in ws]

    a, b = run(True), run(False)
    for x, y in zip(a, b):
        # updates are ~1e-3; bf16 Newton-Schulz may round a few inputs differently
        torch.testing.assert_close(x, y, rtol=1e-3, atol=1e-4)


def test_adamw_table_kernel_matches_torch_adamw_with_ema():
    """One launch for every AdamW parameter (csrc/optim.cu adamw_apply) against torch's fused AdamW over three steps,
    and the EMA moved in the same pass against a separate lerp; the Muon apply with an EMA column likewise."""
    from torch.optim.adam import adam as torch_adam
    from nano_gpic_b200.ops import optim as OPT
    torch.manual_seed(0)
    shapes = [(1024,), (256, 64), (4096,), (32, 48)]
    ps = [torch.randn(s, device="cuda") for s in shapes]
    ref = [p.clone() for p in ps]
    m1, m2 = [torch.zeros_like(p) for p in ps], [torch.zeros_like(p) for p in ps]
    r1, r2 = [torch.zeros_like(p) for p in ps], [torch.zeros_like(p) for p in ps]
    emas = [p.clone() for p in ps]
    ema_ref = [p.clone() for p in ps]
    steps = [torch.zeros((), device="cuda") for _ in ps]
    lr, wd, b1, b2, eps, w = 3e-3, 0.1, 0.9, 0.95, 1e-8, 0.01
    for t in range(1, 4):
        gs = [torch.randn_like(p) for p in ps]
        OPT.adamw_update(ps, gs, m1, m2, emas, lr, wd, b1, b2, eps, 1 - b1 ** t, 1 - b2 ** t, w)
        torch_adam(ref, gs, r1, r2, [], steps, foreach=None, capturable=False, differentiable=False, fused=True,
                   grad_scale=None, found_inf=None, has_complex=False, decoupled_weight_decay=True, amsgrad=False,
                   beta1=b1, beta2=b2, lr=lr, weight_decay=wd, eps=eps, maximize=False)
        for e, r in zip(ema_ref, ref):
            e.lerp_(r, w)
    for a, b in zip(ps, ref):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
    for a, b in zip(m2, r2):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-9)
    for a, b in zip(emas, ema_ref):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
    # Muon apply with the EMA column (rows without an EMA keep theirs untouched)
    P = torch.randn(64, 32, device="cuda")
    O = torch.randn(64, 32, device="cuda").bfloat16()
    E = torch.randn(64, 32, device="cuda")
    P0, E0 = P.clone(), E.clone()
    OPT.apply_updates([(P[:32], O[:32], -0.5, E[:32]), (P[32:], O[32:], 0.25, None)], 0.99, 0.1)
    want = P0 * 0.99 + torch.cat([-0.5 * O[:32].float(), 0.25 * O[32:].float()])
    torch.testing.assert_close(P, want, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(E[:32], E0[:32].lerp(want[:32], 0.1), rtol=1e-6, atol=1e-6)
    assert torch.equal(E[32:], E0[32:])


def test_attached_ema_matches_separate_lerp():
    """MuonAdamW with the EMA attached (the update kernels move it) against the same steps with SimpleEMA's own lerp."""
    from nano_gpic_b200.optim.muon import MuonAdamW
    from nano_gpic_b200.parallel.flat import FlatParams
    from nano_gpic_b200.train.ema import SimpleEMA

    def run(attach):
        torch.manual_seed(2)
        m = torch.nn.Module()
        m.a = torch.nn.Parameter(torch.randn(256, 128, device="cuda") * 0.02)
        m.b = torch.nn.Parameter(torch.randn(384, device="cuda"))
        m.a._muon_parts = 1
        flat = FlatParams(m, device="cuda")
        opt = MuonAdamW(flat.params, lr=1e-3, weight_decay=0.1, muon_lr=2e-2, muon_weight_decay=0.1, split=True)
        ema = SimpleEMA(flat, decay=0.9, off=False)
        if attach:
            assert ema.attach(opt)
        for step in range(1, 4):
            for p in flat.params:
                p.grad = torch.randn_like(p)
            opt.step()
            ema.step(step)
        ema.join()
        return [p.detach().clone() for p in flat.params], ema.buf.clone()

    (pa, ea), (pb, eb) = run(True), run(False)
    for x, y in zip(pa, pb):
        torch.testing.assert_close(x, y, rtol=1e-3, atol=1e-4)
    torch.testing.assert_close(ea, eb, rtol=1e-3, atol=1e-4)


def test_stack_nesterov_with_momentum_update_and_bf16_output():
    """The fused gather: momentum m = lerp(m, g, 1 - beta) written back and the Nesterov input in bf16 in one pass,
    equal to torch's lerp_ then lerp then .to(bfloat16)."""
    from nano_gpic_b200.ops import optim as OPT
    torch.manual_seed(4)
    G = [torch.randn(512, 256, device="cuda") for _ in range(3)]
    M = [torch.randn(512, 256, device="cuda") for _ in range(3)]
    Mr = [m.clone() for m in M]
    for nesterov in (True, False):
        got = OPT.stack_nesterov(G, M, 0.95, nesterov, update_momentum=True, dtype=torch.bfloat16)
        for m, g in zip(Mr, G):
            m.lerp_(g, 1 - 0.95)
        ref = torch.stack([g.lerp(m, 0.95) if nesterov else m for g, m in zip(G, Mr)]).to(torch.bfloat16)
        assert torch.equal(got, ref)
        for a, b in zip(M, Mr):
            assert torch.equal(a, b)


def test_ns_normalize_transpose_and_scale_match_torch():
    """The Newton-Schulz input kernels: X / (||X|| + 1e-7) per matrix in bf16 (optionally transposed) against the
    PyTorch form, the batched transpose exactly, and the clip's in-place scale by a device scalar."""
    from nano_gpic_b200.ops import optim as OPT
    torch.manual_seed(5)
    for n, a, b in ((3, 512, 128), (2, 200, 72), (4, 128, 384)):
        X = (torch.randn(n, a, b, device="cuda") * 3).bfloat16()
        for tr in (False, True):
            Y = X.mT if tr else X
            ref = (Y / (Y.norm(dim=(-2, -1), keepdim=True) + 1e-7)).contiguous()
            got = OPT.ns_normalize(X, transpose=tr)
            assert got.shape == ref.shape and got.is_contiguous()
            torch.testing.assert_close(got.float(), ref.float(), rtol=1e-2, atol=1e-4)
        assert torch.equal(OPT.transpose_bf16(X), X.mT.contiguous())
    buf = torch.randn(1 << 20, device="cuda")
    ref = buf * 0.37
    OPT.scale_(buf, torch.tensor(0.37, device="cuda"))
    assert torch.equal(buf, ref)
