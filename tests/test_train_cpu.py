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


def test_caption_type_losses_and_sinks(tmp_path, monkeypatch):
    """Per-caption-type losses are the per-type means of the step's per-sample losses (0 for an absent type), and the
    sinks write metrics.jsonl and, with a W&B logger configured, log the same values to a (stand-in) wandb run in
    offline mode."""
    import json
    import sys
    import types as pytypes
    from nano_gpic_b200.train.metrics import MetricSinks, caption_type_losses
    per = torch.tensor([1.0, 2.0, 4.0, 8.0, 16.0])
    out = caption_type_losses(per, ["short", "tag", "short", "long", "medium"])
    assert out == {"train/loss_tag": 2.0, "train/loss_short": 2.5, "train/loss_medium": 16.0, "train/loss_long": 8.0}
    assert caption_type_losses(per, [""] * 5)["train/loss_tag"] == 0.0
    calls = []

    class _Run:
        def log(self, values, step):
            calls.append(("log", step, values))

        def finish(self):
            calls.append(("finish",))

    fake = pytypes.ModuleType("wandb")
    fake.init = lambda **kw: calls.append(("init", kw)) or _Run()
    monkeypatch.setitem(sys.modules, "wandb", fake)
    monkeypatch.delenv("WANDB_MODE", raising=False)
    node = {"class_path": "lightning.pytorch.loggers.WandbLogger",
            "init_args": {"name": "ladder", "project": "gpic-speed", "offline": False, "resume": "allow"}}
    sinks = MetricSinks(str(tmp_path), 0, logger_node=node, config={"a": 1})
    monkeypatch.setenv("WANDB_MODE", "offline")
    sinks.log({"loss": 0.5, **out}, 10)
    sinks.close()
    assert calls[0][0] == "init" and calls[0][1]["project"] == "gpic-speed" and calls[0][1]["dir"] == str(tmp_path)
    assert calls[1] == ("log", 10, {"loss": 0.5, **out}) and calls[2] == ("finish",)
    rec = json.loads((tmp_path / "metrics.jsonl").read_text())
    assert rec["step"] == 10 and rec["train/loss_long"] == 8.0
    assert MetricSinks(str(tmp_path), 1, logger_node=node).wandb is None  # only rank 0 writes


def test_prefetch_gives_the_same_steps():
    """Trainer.prefetch (the next step's first micro-batch staged ahead) changes nothing in the steps it feeds, and a
    prefetch of other tensors is ignored."""
    img, cap, mask = _batch()
    img2, cap2, mask2 = _batch(seed=5)
    t = torch.full((4,), 0.3)
    noise = torch.randn(4, 3, 64, 64, generator=torch.Generator().manual_seed(7))
    runs = []
    for use in (False, True):
        tr = _trainer()
        out = []
        for k in range(3):
            a = (img, cap, mask) if k % 2 == 0 else (img2, cap2, mask2)
            out.append(float(tr.train_step(*a, t=t, noise=noise)))
            if use:
                nxt = (img2, cap2, mask2) if k % 2 == 0 else (img, cap, mask)
                tr.prefetch(*nxt, t=t, noise=noise)
        if use:
            tr.prefetch(*_batch(seed=9), t=t, noise=noise)  # not the next step's tensors: ignored
            out.append(float(tr.train_step(img2, cap2, mask2, t=t, noise=noise)))
        else:
            out.append(float(tr.train_step(img2, cap2, mask2, t=t, noise=noise)))
        runs.append(out)
    assert runs[0] == runs[1], runs
