"""The training step on CPU with a tiny model: flat storage, fused objective, clip, Muon/AdamW, schedule."""
import torch


def _trainer(accum=2):
    from nano_gpic_b200.diffusion.flow_matching import JiTTrainer
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    from nano_gpic_b200.optim.lr_scheduler import WarmupFlatCooldown
    from nano_gpic_b200.optim.muon import MuonAdamW, tag_muon_params
    from nano_gpic_b200.parallel.flat import FlatParams
    from nano_gpic_b200.train.trainer import Trainer
    torch.manual_seed(0)
    model = JiT_T2I(input_size=64, in_channels=3, num_groups=2, hidden_size=128, num_blocks=2, num_text_blocks=1,
                    patch_size=16, txt_embed_dim=32, txt_max_length=32, bottleneck_dim=16)
    tag_muon_params(model)
    flat = FlatParams(model)
    opt = MuonAdamW(list(model.parameters()), lr=1e-3, muon_lr=2e-2, split=True, fused_adamw=False,
                    ns_dtype="float32")
    sched = WarmupFlatCooldown(2, 5, 20, min_lr=3e-5)(opt)
    return Trainer(model, opt, sched, JiTTrainer(), accum=accum, clip=1.0, flat=flat)


def _batch(B=4, T=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    img = torch.randint(0, 256, (B, 64, 64, 3), dtype=torch.uint8, generator=g)
    cap = torch.randn(B, T, 32, generator=g).bfloat16()
    mask = torch.arange(T)[None] < torch.randint(1, T + 1, (B,), generator=g)[:, None]
    return img, cap, mask


def test_params_are_flat_views():
    tr = _trainer()
    for p in tr.model.parameters():
        if p.requires_grad:
            assert p.untyped_storage().data_ptr() == tr.flat.data.untyped_storage().data_ptr()
            assert p.grad.untyped_storage().data_ptr() == tr.flat.grad.untyped_storage().data_ptr()


def test_loss_decreases_on_a_fixed_batch():
    tr = _trainer()
    img, cap, mask = _batch()
    t = torch.full((4,), 0.5)
    noise = torch.randn(4, 3, 64, 64, generator=torch.Generator().manual_seed(3))
    losses = [float(tr.train_step(img, cap, mask, t=t, noise=noise)) for _ in range(8)]
    assert losses[-1] < losses[0], losses


def test_accumulation_equals_one_big_batch():
    """Two micro-batches of 2 give the gradient of one batch of 4 (the mean over all images)."""
    img, cap, mask = _batch()
    t = torch.rand(4, generator=torch.Generator().manual_seed(1))
    noise = torch.randn(4, 3, 64, 64, generator=torch.Generator().manual_seed(2))
    grads = []
    for accum in (1, 2):
        tr = _trainer(accum)
        tr.opt.step = lambda: None  # keep the weights: compare the gradients only
        tr.clip = 0
        tr.train_step(img, cap, mask, t=t, noise=noise)
        grads.append(tr.flat.grad.clone())
    rel = (grads[0] - grads[1]).norm() / grads[0].norm()
    assert rel < 2e-2, rel
