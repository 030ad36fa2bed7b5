"""MuonAdamW and WarmupFlatCooldown against the reference's implementations (fp32 Newton-Schulz for exactness)."""
import torch

from refpath import reference_imports


def _params(seed):
    torch.manual_seed(seed)
    m = torch.nn.Module()
    m.blocks = torch.nn.ModuleList([torch.nn.Module()])
    b = m.blocks[0]
    b.attn = torch.nn.Module()
    b.attn.qkv_x = torch.nn.Linear(32, 96, bias=False)
    b.mlp = torch.nn.Module()
    b.mlp.w12 = torch.nn.Linear(32, 256, bias=False)
    b.mlp.w3 = torch.nn.Linear(128, 32, bias=False)
    m.head = torch.nn.Linear(32, 8)
    return m


def test_muon_adamw_matches_reference():
    from nano_gpic_b200.optim.muon import MuonAdamW, tag_muon_params
    with reference_imports():
        from src.optim.muon import MuonAdamW as RefOpt, tag_muon_params as ref_tag
        ref_m = _params(0)
        ref_tag(ref_m)
        ref_opt = RefOpt(list(ref_m.parameters()), lr=1e-3, muon_lr=2e-2, muon_weight_decay=0.01, split=True,
                         fused_adamw=False, ns_dtype="float32")
    m = _params(0)
    tag_muon_params(m)
    opt = MuonAdamW(list(m.parameters()), lr=1e-3, muon_lr=2e-2, muon_weight_decay=0.01, split=True,
                    fused_adamw=False, ns_dtype="float32")
    for step in range(3):
        g = torch.Generator().manual_seed(step)
        for p, q in zip(m.parameters(), ref_m.parameters()):
            gr = torch.randn(p.shape, generator=g)
            p.grad, q.grad = gr.clone(), gr.clone()
        opt.step()
        ref_opt.step()
    for (n, p), q in zip(m.named_parameters(), ref_m.parameters()):
        assert torch.allclose(p, q, atol=1e-6, rtol=1e-5), (n, (p - q).abs().max())
    # the optimizer state dict layout is the reference's
    assert set(opt.state_dict()["state"][0].keys()) == set(ref_opt.state_dict()["state"][0].keys())


def test_warmup_flat_cooldown_matches_reference():
    from nano_gpic_b200.optim.lr_scheduler import WarmupFlatCooldown
    with reference_imports():
        import importlib, sys, types
        sys.modules.setdefault("transformers", importlib.import_module("transformers"))
        from src.utils.lr_scheduler import WarmupFlatCooldown as Ref
    for min_lr in (0.0, 3e-5):
        lrs = []
        for cls in (WarmupFlatCooldown, Ref):
            p = torch.nn.Parameter(torch.zeros(1))
            q = torch.nn.Parameter(torch.zeros(1))
            opt = torch.optim.SGD([{"params": [p], "lr": 1e-3}, {"params": [q], "lr": 1e-2}])
            s = cls(10, 40, 100, min_lr=min_lr)(opt)
            seq = []
            for _ in range(100):
                seq.append([g["lr"] for g in opt.param_groups])
                opt.step()
                s.step()
            lrs.append(seq)
        assert lrs[0] == lrs[1]


def test_adamw_update_fallback_matches_torch_adamw():
    """The PyTorch form of the table kernel (CPU) follows torch.optim.AdamW (decoupled weight decay)."""
    import torch
    from nano_gpic_b200.ops import optim as OPT
    torch.manual_seed(0)
    p = torch.randn(33)  # not a multiple of 4: the PyTorch path
    q = torch.nn.Parameter(p.clone())
    opt = torch.optim.AdamW([q], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    for t in range(1, 5):
        g = torch.randn(33)
        OPT.adamw_update([p], [g], [m], [v], None, 1e-2, 0.1, 0.9, 0.95, 1e-8, 1 - 0.9 ** t, 1 - 0.95 ** t)
        q.grad = g.clone()
        opt.step()
    torch.testing.assert_close(p, q.detach(), rtol=1e-5, atol=1e-6)
