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
