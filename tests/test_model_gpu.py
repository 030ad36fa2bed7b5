"""The model and training step on the GPU kernels against the same code on CPU (fp32 PyTorch op paths)."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

TINY = dict(input_size=64, in_channels=3, num_groups=2, hidden_size=128, num_blocks=2, num_text_blocks=1,
            patch_size=16, txt_embed_dim=32, txt_max_length=32, bottleneck_dim=16)


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-8)).item()


def _model():
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    torch.manual_seed(0)
    m = JiT_T2I(**TINY)
    with torch.no_grad():
        for p in m.parameters():
            if p.requires_grad:
                p.add_(torch.randn_like(p) * 0.05)
    return m


def test_model_forward_backward_cuda_vs_cpu():
    cpu = _model()
    gpu = copy.deepcopy(cpu).cuda()
    g = torch.Generator().manual_seed(1)
    x = torch.rand(4, 3, 64, 64, generator=g) * 2 - 1
    t = torch.rand(4, generator=g)
    y = torch.randn(4, 24, 32, generator=g)
    mask = torch.arange(24)[None] < torch.tensor([24, 3, 17, 9])[:, None]
    oc = cpu(x, t, y, y_mask=mask)
    og = gpu(x.cuda(), t.cuda(), y.cuda(), y_mask=mask.cuda())
    assert _rel(og, oc) < 2e-2
    w = torch.randn_like(oc)
    (oc * w).sum().backward()
    (og * w.cuda()).sum().backward()
    for (n, pc), pg in zip(cpu.named_parameters(), gpu.parameters()):
        if pc.requires_grad:
            assert _rel(pg.grad, pc.grad) < 5e-2, n
    from nano_gpic_b200.ops import status
    assert status.read() == 0


def test_elementwise_ops():
    from nano_gpic_b200.ops import elementwise as E
    g = torch.Generator().manual_seed(0)
    x = torch.rand(3, 3, 64, 64, generator=g) * 2 - 1
    n = torch.randn(3, 3, 64, 64, generator=g)
    t = torch.rand(3, generator=g)
    tok_c = E.fm_prep(x, n, t, 16)
    tok_g = E.fm_prep(x.cuda(), n.cuda(), t.cuda(), 16)
    assert _rel(tok_g, tok_c) < 1e-2
    pred = torch.randn(3 * 16, 768, generator=g).bfloat16()
    pc, gc = E.fm_loss(pred, x, n, t, 16)
    pg, gg = E.fm_loss(pred.cuda(), x.cuda(), n.cuda(), t.cuda(), 16)
    assert _rel(pg, pc) < 1e-4 and _rel(gg, gc) < 1e-2
    img = E.unpatchify(pred.cuda(), 3, 3, 64, 64, 16)
    assert _rel(img, E.unpatchify(pred, 3, 3, 64, 64, 16)) < 1e-6
    assert _rel(E.patchify(img, 16), pred) < 1e-2
    a = torch.randn(48, 128, generator=g).bfloat16()
    tab = torch.randn(16, 128, generator=g)
    assert _rel(E.add_rows(a.cuda(), tab.cuda(), 16), E.add_rows(a, tab, 16)) < 1e-2
    dout, yv = torch.randn(48, 128, generator=g).bfloat16(), torch.randn(48, 128, generator=g).bfloat16()
    gate = torch.randn(3, 768, generator=g).bfloat16()[:, 128:256]
    dgc, dbc = torch.zeros(3, 128), torch.zeros(128)
    dyc = E.gate_bwd(dout, yv, gate, 16, dgc, dbc)
    dgg, dbg = torch.zeros(3, 128, device="cuda"), torch.zeros(128, device="cuda")
    dyg = E.gate_bwd(dout.cuda(), yv.cuda(), gate.cuda(), 16, dgg, dbg)
    assert _rel(dyg, dyc) < 1e-2 and _rel(dgg, dgc) < 1e-3 and _rel(dbg, dbc) < 1e-3


def test_msign_bf16_kernel_vs_fp32():
    from nano_gpic_b200.optim.muon import msign
    G = torch.randn(3, 512, 128, device="cuda")
    ref = msign(G, dtype=torch.float32)
    out = msign(G, dtype=torch.bfloat16)
    # bf16 Newton-Schulz moves entries by a few percent (reference muon.py:67-68)
    assert _rel(out, ref) < 0.1
    assert out.shape == G.shape


def test_trainer_steps_on_gpu():
    from nano_gpic_b200.diffusion.flow_matching import JiTTrainer
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    from nano_gpic_b200.ops import status
    from nano_gpic_b200.optim.lr_scheduler import WarmupFlatCooldown
    from nano_gpic_b200.optim.muon import MuonAdamW, tag_muon_params
    from nano_gpic_b200.parallel.flat import FlatParams
    from nano_gpic_b200.train.trainer import Trainer
    torch.manual_seed(0)
    model = JiT_T2I(**TINY).cuda()
    tag_muon_params(model)
    flat = FlatParams(model)
    opt = MuonAdamW(list(model.parameters()), lr=1e-3, muon_lr=2e-2, split=True)
    tr = Trainer(model, opt, WarmupFlatCooldown(1, 5, 20)(opt), JiTTrainer(), accum=2, flat=flat)
    g = torch.Generator().manual_seed(0)
    img = torch.randint(0, 256, (8, 64, 64, 3), dtype=torch.uint8, generator=g).cuda()
    cap = torch.randn(8, 16, 32, generator=g).bfloat16().cuda()
    mask = (torch.arange(16)[None] < torch.randint(1, 17, (8,), generator=g)[:, None]).cuda()
    t = torch.full((8,), 0.5, device="cuda")
    noise = torch.randn(8, 3, 64, 64, device="cuda")
    losses = [float(tr.train_step(img, cap, mask, t=t, noise=noise)) for _ in range(6)]
    assert all(torch.isfinite(torch.tensor(losses))), losses
    assert losses[-1] < losses[0], losses
    assert status.read() == 0


@pytest.mark.parametrize("C", [1024, 768, 1280])
def test_gate_bwd_model_widths(C):
    """gate_bwd at the model's widths (two row groups per block at C <= 1024, one above) against the CPU path."""
    from nano_gpic_b200.ops import elementwise as E
    g = torch.Generator().manual_seed(C)
    M, rpg = 3 * 256, 256
    G = (M + rpg - 1) // rpg
    dout, yv = torch.randn(M, C, generator=g).bfloat16(), torch.randn(M, C, generator=g).bfloat16()
    gate = torch.randn(G, 3 * C, generator=g).bfloat16()[:, C:2 * C]
    dgc, dbc = torch.zeros(G, C), torch.zeros(C)
    dyc = E.gate_bwd(dout, yv, gate, rpg, dgc, dbc)
    dgg, dbg = torch.zeros(G, C, device="cuda"), torch.zeros(C, device="cuda")
    dyg = E.gate_bwd(dout.cuda(), yv.cuda(), gate.cuda(), rpg, dgg, dbg)
    assert _rel(dyg, dyc) < 1e-2 and _rel(dgg, dgc) < 1e-3 and _rel(dbg, dbc) < 1e-3
