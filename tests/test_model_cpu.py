"""JiT-T2I on the framework's ops (CPU paths) against the reference's own JiT_T2I module: state-dict keys, forward
output and every parameter gradient, on a tiny configuration with random (non-zero) weights."""
import pytest
import torch

from refpath import reference_imports

TINY = dict(input_size=64, in_channels=3, num_groups=2, hidden_size=128, num_blocks=2, num_text_blocks=1,
            patch_size=16, txt_embed_dim=32, txt_max_length=32, bottleneck_dim=16)


def _models(seed=0):
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    with reference_imports():
        from src.models.transformer.JiT_T2I import JiT_T2I as Ref
        torch.manual_seed(seed)
        ref = Ref(**TINY)
    with torch.no_grad():
        for p in ref.parameters():
            if p.requires_grad:
                p.copy_(torch.randn_like(p) * (0.2 if p.ndim == 2 else 0.05) + (1.0 if p.ndim == 1 and p.numel() in
                                                                                   (64, 128) else 0.0))
    ours = JiT_T2I(**TINY)
    ours.load_state_dict(ref.state_dict(), strict=True)
    return ref, ours


def _inputs(B=2, T=16, seed=1):
    g = torch.Generator().manual_seed(seed)
    x = torch.rand(B, 3, 64, 64, generator=g) * 2 - 1
    t = torch.rand(B, generator=g)
    y = torch.randn(B, T, 32, generator=g)
    lens = torch.tensor([T, 5])[:B]
    mask = torch.arange(T)[None] < lens[:, None]
    return x, t, y, mask


def test_state_dict_keys_match():
    ref, ours = _models()
    assert list(ref.state_dict().keys()) == list(ours.state_dict().keys())
    for k, v in ref.state_dict().items():
        assert ours.state_dict()[k].shape == v.shape, k


def test_forward_and_grads_match_reference():
    """Our bf16 kernels' error against the fp32 reference must stay within 2x the reference's own error when it runs
    under bf16 autocast (its training precision), per output and per parameter gradient."""
    ref, ours = _models()
    x, t, y, mask = _inputs()
    w = None
    grads = {}
    outs = {}
    for name, amp in (("fp32", False), ("bf16", True)):
        ref.zero_grad()
        with torch.autocast("cpu", dtype=torch.bfloat16, enabled=amp):
            o = ref(x, t, y, y_mask=mask)
        if w is None:
            w = torch.randn_like(o.float())
        (o.float() * w).sum().backward()
        outs[name] = o.float().detach()
        grads[name] = {n: p.grad.clone() for n, p in ref.named_parameters() if p.grad is not None}
    out = ours(x, t, y, y_mask=mask)
    (out.float() * w).sum().backward()

    def rel(a, b):
        return (a - b).norm().item() / (b.norm().item() + 1e-8)
    e_ours, e_amp = rel(out.float(), outs["fp32"]), rel(outs["bf16"], outs["fp32"])
    assert e_ours <= max(2 * e_amp, 1e-2), (e_ours, e_amp)
    bad = []
    for n, p in ours.named_parameters():
        if not p.requires_grad:
            continue
        assert p.grad is not None, n
        e1, e2 = rel(p.grad, grads["fp32"][n]), rel(grads["bf16"][n], grads["fp32"][n])
        if e1 > max(2 * e2, 2e-2):
            bad.append((n, round(e1, 4), round(e2, 4)))
    assert not bad, bad


def test_recompute_matches_stored_activations():
    """Activation checkpointing reruns each block's forward in the backward: same output and gradients, bit for bit."""
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    torch.manual_seed(0)
    net = JiT_T2I(input_size=32, in_channels=3, num_groups=2, hidden_size=128, num_blocks=2, num_text_blocks=1,
                  patch_size=16, txt_embed_dim=2048, txt_max_length=8)
    with torch.no_grad():
        for prm in net.parameters():
            prm.add_(torch.randn_like(prm) * 0.02)
    x, t = torch.randn(2, 3, 32, 32), torch.rand(2)
    y = torch.randn(2, 8, 2048).to(torch.bfloat16)
    m = torch.ones(2, 8, dtype=torch.bool)
    m[1, 5:] = False
    res = []
    for mode in (None, "all"):
        net.set_recompute(mode)
        net.zero_grad(set_to_none=True)
        o = net(x, t, y, y_mask=m)
        o.float().square().mean().backward()
        res.append((o.detach().clone(), [p.grad.clone() for p in net.parameters() if p.grad is not None]))
    assert torch.equal(res[0][0], res[1][0])
    assert len(res[0][1]) == len(res[1][1])
    for a, b in zip(res[0][1], res[1][1]):
        assert torch.equal(a, b)
