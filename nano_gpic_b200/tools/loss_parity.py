"""Loss parity at equal steps: this framework against the reference's own modules, from the same initial weights, on
the same batches, timesteps and noise, scored by the fixed-noise held-out loss over 16 levels.

    python -m nano_gpic_b200.tools.loss_parity --size d12 --steps 40 --batch 256 [--fp8 mx] --out parity.json

* Weights: this framework's initial state dict is loaded into the reference's JiT_T2I (the keys are the same).
* Training: ours through `Trainer.train_step`; the reference through its JiTTrainer under bf16 autocast, its MuonAdamW
  (split, bf16 Newton-Schulz, mup scale), WarmupFlatCooldown and global-norm clip 1.0 (the ladder recipe, reference
  jobs/final_ladder.sh and configs_h100/lite_ladder.yaml), eager. Its JiTTrainer draws t (`randn(B)`, logit-normal)
  and then the noise (`randn_like(x)`) from the global generator (training_JiT.py:36-47); seeding that generator before
  each micro-batch and drawing the same two tensors for ours gives both runs the same t and noise.
* Data: synthetic uint8 images and N(0, 1) caption features with random-length left-aligned masks, one seed per step.
* Score: the held-out loss of tools/heldout_loss (16 logit-normal quantile levels, fixed noise per image and level) on
  a held-out synthetic set, before and after training; the figure of merit is |ours - ref| / ref after training.
"""
import argparse
import json
import os
import sys
import time

import torch

from ..config.ladder import SIZES
from .heldout_loss import image_noise, level_loss, levels, time_shift_fn

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def batch(seed, B, T, device):
    g = torch.Generator().manual_seed(seed)
    img = torch.randint(0, 256, (B, 256, 256, 3), dtype=torch.uint8, generator=g)
    cap = torch.randn(B, T, 2048, generator=g).to(torch.bfloat16)
    lens = torch.randint(8, T + 1, (B,), generator=g)
    mask = torch.arange(T)[None, :] < lens[:, None]
    return img.to(device), cap.to(device), mask.to(device)


def to_float(u8):
    """ToTensor + Normalize(0.5, 0.5) of the reference's train transform, [B, H, W, 3] uint8 -> [B, 3, H, W]."""
    return ((u8.permute(0, 3, 1, 2).float() / 255.0) - 0.5) / 0.5


def draws(seed, mb, device, P_mean=-0.8, P_std=0.8):
    """The reference JiTTrainer's two draws after seeding the global generator: t (logit-normal) and the noise."""
    torch.manual_seed(seed)
    t = time_shift_fn((torch.randn(mb, device=device, dtype=torch.float32) * P_std + P_mean).sigmoid(), 1.0)
    noise = torch.randn(mb, 3, 256, 256, device=device, dtype=torch.float32)
    return t, noise


@torch.no_grad()
def heldout(net, data, ts, seed, autocast):
    img, cap, mask = data
    x = to_float(img)
    per_level = []
    for j, t in enumerate(ts):
        noise = image_noise(seed, j, 1, tuple(x.shape))[0].to(x.device)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            per_level.append(level_loss(net, x, cap, mask, t.to(x.device), noise).mean().item())
    return sum(per_level) / len(per_level), per_level


def reference_parts(size, device, ref_root, warmup=None):
    pg = os.path.join(ref_root, "baselines", "PixelGen")
    if not os.path.isdir(os.path.join(pg, "src")):
        raise SystemExit(f"reference tree not found under {ref_root}")
    os.environ.setdefault("GPIC_MFU_ATTN", "sdpa")  # FA3 is a Hopper-only binary
    os.environ.setdefault("GPIC_MFU_FUSED_NORM", "1")
    os.environ.setdefault("GPIC_MFU_NS_FUSED", "1")
    os.environ.setdefault("GPIC_MFU_MUON_ADD", "1")
    sys.path.insert(0, pg)
    from src.diffusion.flow_matching.scheduling import LinearScheduler
    from src.diffusion.flow_matching.training_JiT import JiTTrainer, constant
    from src.models.transformer.JiT_T2I import JiT_T2I
    from src.optim.muon import MuonAdamW, tag_muon_params
    from src.utils.lr_scheduler import WarmupFlatCooldown
    s = SIZES[size]
    net = JiT_T2I(**s.model_kwargs()).to(device)
    tag_muon_params(net)
    params = [p for p in net.parameters() if p.requires_grad]
    opt = MuonAdamW([{"params": params}], lr=s.adamw_lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0,
                    muon_lr=s.muon_lr, muon_weight_decay=s.muon_wd, muon_momentum=0.95, muon_nesterov=True, ns_steps=5,
                    split=True, fused_adamw=True, ns_dtype="bfloat16", update_scale="mup")
    wu, cd = s.schedule()
    sched = WarmupFlatCooldown(wu if warmup is None else warmup, cd, s.steps, min_lr=3e-5)(opt)
    obj = JiTTrainer(scheduler=LinearScheduler(), loss_weight_fn=constant, lognorm_t=True, timeshift=1.0, P_mean=-0.8,
                     P_std=0.8, t_eps=0.05, null_condition_p=0.0)
    return net, params, opt, sched, obj


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--size", default="d12")
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--batch", type=int, default=256, help="images per optimizer step")
    ap.add_argument("--micro-batch", type=int, default=128)
    ap.add_argument("--caption-len", type=int, default=128)
    ap.add_argument("--heldout", type=int, default=64, help="held-out images")
    ap.add_argument("--fp8", default="none", choices=["none", "mx", "mx2"], help="our arm's GEMM precision")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--lr-warmup", type=int, default=None,
                    help="warmup steps of both schedules (default: the ladder's, 1%% of the full run)")
    ap.add_argument("--ref-root", default=os.path.join(ROOT, "baseline", "_ref"))
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    dev = torch.device("cuda")
    from ..train.trainer import Trainer
    tr = Trainer.for_ladder(a.size, device=dev, micro_batch=a.micro_batch, global_batch=a.batch, dp="ddp",
                            seed=a.seed, fp8=None if a.fp8 == "none" else a.fp8)
    if a.lr_warmup is not None:
        from ..optim.lr_scheduler import WarmupFlatCooldown
        s = SIZES[a.size]
        tr.sched = WarmupFlatCooldown(a.lr_warmup, s.schedule()[1], s.steps, min_lr=3e-5)(tr.opt)
    ref, rparams, ropt, rsched, robj = reference_parts(a.size, dev, a.ref_root, a.lr_warmup)
    ref.load_state_dict(tr.model.state_dict(), strict=True)
    ts = levels()
    held = batch(10_000 + a.seed, a.heldout, a.caption_len, dev)
    rec = {"size": a.size, "steps": a.steps, "lr_warmup": a.lr_warmup, "batch": a.batch, "micro_batch": a.micro_batch, "fp8": a.fp8,
           "caption_len": a.caption_len, "heldout_images": a.heldout, "levels": [round(float(t), 5) for t in ts]}
    rec["heldout_init"] = {"ours": heldout(tr.model, held, ts, a.seed, False)[0],
                           "reference": heldout(ref, held, ts, a.seed, True)[0]}
    accum = a.batch // a.micro_batch
    train = {"ours": [], "reference": []}
    t0 = time.time()
    for step in range(a.steps):
        img, cap, mask = batch(a.seed * 1_000_003 + step, a.batch, a.caption_len, dev)
        ts_, ns_ = [], []
        for i in range(accum):
            t, n = draws(a.seed * 7919 + step * 101 + i, a.micro_batch, dev)
            ts_.append(t)
            ns_.append(n)
        train["ours"].append(float(tr.train_step(img, cap, mask, t=torch.cat(ts_), noise=torch.cat(ns_))))
        losses = []
        for i in range(accum):
            sl = slice(i * a.micro_batch, (i + 1) * a.micro_batch)
            torch.manual_seed(a.seed * 7919 + step * 101 + i)  # the same t and noise draws (see draws())
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = robj(ref, None, None, to_float(img[sl]), cap[sl], None, {"y_mask": mask[sl]})
            (out["loss"] / accum).backward()
            losses.append(out["loss"].detach())
        torch.nn.utils.clip_grad_norm_(rparams, 1.0, foreach=True)
        ropt.step()
        rsched.step()
        ropt.zero_grad(set_to_none=True)
        train["reference"].append(float(torch.stack(losses).mean()))
    rec["train_seconds"] = round(time.time() - t0, 1)
    rec["train_loss"] = {k: [round(v, 6) for v in vs] for k, vs in train.items()}
    o, o_lv = heldout(tr.model, held, ts, a.seed, False)
    r, r_lv = heldout(ref, held, ts, a.seed, True)
    rec["heldout_final"] = {"ours": o, "reference": r, "ours_levels": o_lv, "reference_levels": r_lv}
    rec["rel_diff_final"] = abs(o - r) / r
    rec["within_0.5pct"] = rec["rel_diff_final"] <= 0.005
    line = json.dumps(rec)
    print(line, flush=True)
    if a.out:
        with open(a.out, "w") as f:
            f.write(line + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
