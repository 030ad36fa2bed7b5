#!/usr/bin/env python
"""Headline benchmark: training images/s of the whole job (and MFU) on ladder JiT-T2I d12, global batch 1024,
256x256 images, 128-token captions of 2048-d features with random-length masks (synthetic data, random init).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--size d12] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

One optimizer step = 1024 images over all ranks (1024 / N per rank, split into micro-batches of 128). Timing: W
untimed warm-up steps, then exactly K steps bracketed by a barrier + cuda synchronize on both sides, timed with CUDA
events on the launching stream; the reported time is the max over ranks. Every step's inputs (about 1.3 GB per rank)
exceed the 126 MB L2. `e2e` repeats the measurement through the public Trainer.train_step API with each step's inputs
copied from pinned host memory and every step's loss read back to the host (one step behind, while the next step
runs; the last read closes the timed region), for both arms; ours also starts each step's first host -> device copy
under the previous step (Trainer.prefetch). `--impl reference` runs the unmodified reference
(baseline/_ref: its JiT_T2I, JiTTrainer, MuonAdamW, WarmupFlatCooldown, bf16 autocast, SDPA attention because its FA3
binary is Hopper-only) on the same data, with the data parallelism its final ladder uses for the size: whole-model
torch.compile + DDP below width 1280, FSDP2 per block + ShardMuonAdamW + NoSync accumulation from width 1280 (d14+)
on more than one GPU (its sharded optimizer does not run on one GPU, where it trains unsharded).
`parallelism` names the work (dpN: N data-parallel ranks over one global batch) and is the same for both arms;
`dp_mode` says how each arm carries it out.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
PUBLISHED = {"d12": 7817.0, "d18": 2183.0, "d10": 12724.0}  # the reference's published images/s per 8 x H100 box


# ------------------------------------------------------------------------------------------------------- helpers
def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"] * 1e12, "measured"
    return 1590e12, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons every 200 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r for r in self.rows if r[0].isdigit() and int(r[0]) in self.gpus]
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        mx = max((float(r[2]) for r in rows if r[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


def synthetic_batch(B, T, D, seed, device="cpu", pin=False):
    """uint8 images [B, 256, 256, 3] (uniform, i.e. x uniform in [-1, 1]), caption features N(0, 1) bf16 [B, T, D],
    left-aligned masks with lengths uniform in [1, T] (the longest padded to T)."""
    g = torch.Generator().manual_seed(seed)
    img = torch.randint(0, 256, (B, 256, 256, 3), dtype=torch.uint8, generator=g)
    cap = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    lens = torch.randint(1, T + 1, (B,), generator=g)
    lens[0] = T
    mask = torch.arange(T)[None] < lens[:, None]
    out = [img, cap, mask]
    if pin:
        out = [t.pin_memory() for t in out]
    if device != "cpu":
        out = [t.to(device) for t in out]
    return out


def max_over_ranks(v, device):
    t = torch.tensor([v], dtype=torch.float64, device=device)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sync_all():
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()


def timed_e2e(step_fn, K):
    """Like timed() for the end-to-end run: step_fn(i) runs step i from host inputs and returns its loss (a device
    scalar); every step's loss is read back to the host, one step behind (while the next step runs, as a training loop
    that logs asynchronously does), and the last step's read is inside the timed region."""
    sync_all()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    prev, vals = None, []
    for i in range(K):
        loss = step_fn(i)
        if prev is not None:
            vals.append(prev.item())
        prev = loss
    vals.append(prev.item())
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    sync_all()
    assert len(vals) == K
    return ms


def timed(step_fn, K):
    sync_all()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        step_fn(i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    sync_all()
    return ms


# ------------------------------------------------------------------------------------------------------- our arm
def run_ours(a, rank, world, dev):
    from nano_gpic_b200 import _ext
    from nano_gpic_b200.ops import status
    from nano_gpic_b200.train.trainer import Trainer
    tr = Trainer.for_ladder(a.size, device=dev, world=world, rank=rank, micro_batch=a.micro_batch, dp=a.dp,
                            transport=a.transport, fp8=None if a.fp8 == "none" else a.fp8,
                            recompute=None if a.recompute == "none" else a.recompute,
                            global_batch=a.global_batch)
    B = a.global_batch // world
    dev_batch = synthetic_batch(B, a.caption_len, 2048, seed=1000 + rank, device=dev)
    host_batches = [synthetic_batch(B, a.caption_len, 2048, seed=2000 + 10 * rank + i, pin=True) for i in range(2)]

    def dev_step(i):
        return tr.train_step(*dev_batch)

    for _ in range(a.warmup):
        dev_step(0)
    torch.cuda.synchronize()
    status.check()
    l0 = _ext.ext().launch_count()
    clocks = ClockSampler(range(world) if rank == 0 else []) if rank == 0 else None
    if clocks:
        clocks.start()
    ms = timed(dev_step, a.steps)
    launches = _ext.ext().launch_count() - l0
    clock_rec = clocks.stop() if clocks else None
    status.check()
    e2e_ms = None
    if not a.no_e2e:
        def e2e_step(i):
            loss = tr.train_step(*host_batches[i % 2])
            tr.prefetch(*host_batches[(i + 1) % 2])  # the next step's first copies run under this step
            return loss
        e2e_ms = timed_e2e(e2e_step, a.steps)
    return ms, e2e_ms, launches, clock_rec, tr


# ------------------------------------------------------------------------------------------------- reference arm
def reference_step_fn(a, rank, world, dev):
    """The reference's training step (one optimizer step over this rank's batch), built from its own classes."""
    pg = os.path.join(ROOT, "baseline", "_ref", "baselines", "PixelGen")
    # the reference's final-ladder levers for a DDP size (jobs/final_ladder.sh:30-35), minus FA3 (Hopper-only binary)
    os.environ.setdefault("GPIC_MFU_ATTN", "sdpa")
    os.environ.setdefault("GPIC_MFU_FUSED_NORM", "1")
    os.environ.setdefault("GPIC_MFU_NS_FUSED", "1")
    os.environ.setdefault("GPIC_MFU_MUON_ADD", "1")
    os.environ.setdefault("GPIC_MFU_NO_EMA", "1")
    sys.path.insert(0, pg)
    from src.diffusion.flow_matching.scheduling import LinearScheduler
    from src.diffusion.flow_matching.training_JiT import JiTTrainer, constant
    from src.models.transformer.JiT_T2I import JiT_T2I
    from src.optim.muon import MuonAdamW, tag_muon_params
    from src.utils.lr_scheduler import WarmupFlatCooldown
    from nano_gpic_b200.config.ladder import SIZES
    s = SIZES[a.size]
    torch.set_float32_matmul_precision("medium")  # reference patch_bugs.py:5
    torch.manual_seed(0)
    net = JiT_T2I(**s.model_kwargs()).to(dev)
    # the reference caches its RoPE tables on first use; building them eagerly keeps that CPU work out of the compiled
    # graph (as its own compile warm-up does), so Inductor emits GPU kernels only
    net.fetch_pos(256 // 16, 256 // 16, dev)
    tag_muon_params(net)
    params = [p for p in net.parameters() if p.requires_grad]
    opt = MuonAdamW([{"params": params}], lr=s.adamw_lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0,
                    muon_lr=s.muon_lr, muon_weight_decay=s.muon_wd, muon_momentum=0.95, muon_nesterov=True, ns_steps=5,
                    split=True, fused_adamw=True, ns_dtype="bfloat16", update_scale="mup")
    wu, cd = s.schedule()
    sched = WarmupFlatCooldown(wu, cd, s.steps, min_lr=3e-5)(opt)
    model = net
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(net, device_ids=[dev.index], broadcast_buffers=False,
                                                          gradient_as_bucket_view=True, bucket_cap_mb=1000)
    model = torch.compile(model)
    trainer = JiTTrainer(scheduler=LinearScheduler(), loss_weight_fn=constant, lognorm_t=True, timeshift=1.0,
                         P_mean=-0.8, P_std=0.8, t_eps=0.05, null_condition_p=0.0)
    mb = a.micro_batch or s.micro_batch
    B = a.global_batch // world
    accum = B // mb

    def to_float(u8):  # ToTensor + Normalize(0.5, 0.5) of the reference's train transform
        return ((u8.permute(0, 3, 1, 2).float() / 255.0) - 0.5) / 0.5

    def step(img, cap, mask):
        losses = []
        for i in range(accum):
            sl = slice(i * mb, (i + 1) * mb)
            x = to_float(img[sl].to(dev, non_blocking=True))
            y = cap[sl].to(dev, non_blocking=True)
            m = mask[sl].to(dev, non_blocking=True)
            ctx = model.no_sync() if (world > 1 and i < accum - 1 and hasattr(model, "no_sync")) else None
            with torch.autocast("cuda", dtype=torch.bfloat16):
                if ctx is not None:
                    with ctx:
                        out = trainer(model, None, None, x, y, None, {"y_mask": m})
                        (out["loss"] / accum).backward()
                else:
                    out = trainer(model, None, None, x, y, None, {"y_mask": m})
                    (out["loss"] / accum).backward()
            losses.append(out["loss"].detach())
        torch.nn.utils.clip_grad_norm_(params, 1.0, foreach=True)
        opt.step()
        sched.step()
        opt.zero_grad(set_to_none=True)
        return torch.stack(losses).mean()

    return step


FSDP_WIDTH = 1280  # the reference's final ladder runs FSDP2 from this width up, DDP below (jobs/final_ladder.sh:29-30)


def reference_uses_fsdp(size, world):
    """FSDP2 for the reference's FSDP sizes on more than one GPU. On one GPU its ShardMuonAdamW hands the step to the
    unsharded MuonAdamW (muon_fsdp.py:93-94), which cannot take FSDP2's DTensor parameters, so a 1-GPU run of the
    reference is its unsharded path (whole-model compile, no wrapper), as for the DDP sizes."""
    from nano_gpic_b200.config.ladder import SIZES
    return SIZES[size].width >= FSDP_WIDTH and world > 1


def reference_fsdp_step_fn(a, rank, world, dev):
    """The reference's FSDP2 training step for its FSDP sizes (d14 and up), built from its own code as its Lightning
    path does: fsdp_setup.shard (one fully_shard unit per block, or groups of 7 blocks at width 1280; bf16 compute
    parameters, fp32 reduce; RMSNorm weights and pos_embed replicated; each block compiled), MuonAdamW turned into
    ShardMuonAdamW.like (owner all-to-alls around Newton-Schulz), replicated-gradient all-reduce, the global-norm clip
    over DTensor shards, and NoSync accumulation (no reduce-scatter before the last micro-batch). The levers are those
    of jobs/final_ladder.sh:29-35 for an FSDP size, minus FA3 (a Hopper-only binary)."""
    pg = os.path.join(ROOT, "baseline", "_ref", "baselines", "PixelGen")
    from nano_gpic_b200.config.ladder import SIZES
    s = SIZES[a.size]
    os.environ.setdefault("GPIC_MFU_ATTN", "sdpa")
    for k in ("GPIC_MFU_FSDP", "GPIC_MFU_FSDP_NOSYNC", "GPIC_MFU_LOCAL_OPT", "GPIC_MFU_PATCHIFY", "GPIC_MFU_FUSED_NORM",
              "GPIC_MFU_FUSED_QK", "GPIC_MFU_NS_FUSED", "GPIC_MFU_MUON_ADD", "GPIC_MFU_NO_EMA"):
        os.environ.setdefault(k, "1")
    os.environ.setdefault("GPIC_MFU_FSDP_GROUP", "7" if s.width == 1280 else "1")
    sys.path.insert(0, pg)
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.fsdp import FSDPModule
    from src.diffusion.flow_matching.scheduling import LinearScheduler
    from src.diffusion.flow_matching.training_JiT import JiTTrainer, constant
    from src.models.transformer.JiT_T2I import JiT_T2I
    from src.optim.muon import MuonAdamW, tag_muon_params
    from src.optim.muon_fsdp import ShardMuonAdamW
    from src.utils.fsdp_setup import clip_grad_norm_, is_dtensor, shard, sync_replicated_grads
    from src.utils.lr_scheduler import WarmupFlatCooldown
    torch.set_float32_matmul_precision("medium")  # reference patch_bugs.py:5
    torch.manual_seed(0)
    net = JiT_T2I(**s.model_kwargs()).to(dev)
    net.fetch_pos(256 // 16, 256 // 16, dev)
    mesh = init_device_mesh("cuda", (world,))
    replicated = shard(net, mesh, compute_bf16=True, compile_blocks=True)
    tag_muon_params(net)  # after sharding, as its configure_optimizers runs after configure_model
    params = [p for p in net.parameters() if p.requires_grad]
    groups = [{"params": [p for p in params if is_dtensor(p)]}, {"params": [p for p in params if not is_dtensor(p)]}]
    opt = MuonAdamW(groups, lr=s.adamw_lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, muon_lr=s.muon_lr,
                    muon_weight_decay=s.muon_wd, muon_momentum=0.95, muon_nesterov=True, ns_steps=5, split=True,
                    fused_adamw=True, ns_dtype="bfloat16", update_scale="mup")
    opt = ShardMuonAdamW.like(opt, groups)
    wu, cd = s.schedule()
    sched = WarmupFlatCooldown(wu, cd, s.steps, min_lr=3e-5)(opt)
    units = [m for m in net.modules() if isinstance(m, FSDPModule)]
    trainer = JiTTrainer(scheduler=LinearScheduler(), loss_weight_fn=constant, lognorm_t=True, timeshift=1.0,
                         P_mean=-0.8, P_std=0.8, t_eps=0.05, null_condition_p=0.0)
    mb = a.micro_batch or s.micro_batch
    accum = (a.global_batch // world) // mb

    def to_float(u8):
        return ((u8.permute(0, 3, 1, 2).float() / 255.0) - 0.5) / 0.5

    def sync(on):  # NoSyncModelParallelStrategy.block_backward_sync
        for m in units:
            m.set_requires_gradient_sync(on, recurse=False)
            m.set_reshard_after_backward(on, recurse=False)

    def step(img, cap, mask):
        losses = []
        for i in range(accum):
            sl = slice(i * mb, (i + 1) * mb)
            x = to_float(img[sl].to(dev, non_blocking=True))
            y = cap[sl].to(dev, non_blocking=True)
            m = mask[sl].to(dev, non_blocking=True)
            sync(i == accum - 1)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = trainer(net, None, None, x, y, None, {"y_mask": m})
                (out["loss"] / accum).backward()
            losses.append(out["loss"].detach())
        sync_replicated_grads(replicated)
        clip_grad_norm_(params, 1.0)
        opt.step()
        sched.step()
        opt.zero_grad(set_to_none=True)
        return torch.stack(losses).mean()

    return step


def run_reference(a, rank, world, dev):
    pg = os.path.join(ROOT, "baseline", "_ref", "baselines", "PixelGen")
    if not os.path.isdir(os.path.join(pg, "src")):
        return None, "baseline/_ref is missing: copy the reference source tree there (cp -r; it is not a pip package)"
    fsdp = reference_uses_fsdp(a.size, world)
    step = (reference_fsdp_step_fn if fsdp else reference_step_fn)(a, rank, world, dev)
    B = a.global_batch // world
    dev_batch = synthetic_batch(B, a.caption_len, 2048, seed=1000 + rank, device=dev)
    host_batches = [synthetic_batch(B, a.caption_len, 2048, seed=2000 + 10 * rank + i, pin=True) for i in range(2)]
    for _ in range(a.warmup):
        step(*dev_batch)
    torch.cuda.synchronize()
    clocks = ClockSampler(range(world)) if rank == 0 else None
    if clocks:
        clocks.start()
    ms = timed(lambda i: step(*dev_batch), a.steps)
    clock_rec = clocks.stop() if clocks else None
    e2e_ms = None
    if not a.no_e2e:
        e2e_ms = timed_e2e(lambda i: step(*host_batches[i % 2]), a.steps)
    return (ms, e2e_ms, None, clock_rec, None), None


# ---------------------------------------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--size", default="d12")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--micro-batch", type=int, default=None)
    ap.add_argument("--global-batch", type=int, default=1024)
    ap.add_argument("--caption-len", type=int, default=128)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--recompute", default="none", choices=["none", "image", "all"],
                    help="activation checkpointing of the image (and text) blocks")
    ap.add_argument("--fp8", default="none", choices=["none", "mx", "mx2"],
                    help="mx: the image blocks' forward GEMMs in MXFP8 (the d12-FP8 config); mx2: also the MLP dgrads "
                         "(the reference's phase 2); default bf16")
    ap.add_argument("--transport", default="nccl", choices=["nccl", "p2p"],
                    help="zero mode: NCCL collectives or this framework's peer-memory kernels")
    ap.add_argument("--dp", default="zero", choices=["ddp", "zero"],
                    help="data-parallel mode of our arm: all-reduce (the reference's DDP sizes) or reduce-scatter to "
                         "owners with sharded optimizer state (its FSDP2 sizes)")
    a = ap.parse_args()
    assert a.warmup >= 3, "at least 3 warm-up steps"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world == a.gpus, f"--gpus {a.gpus} but WORLD_SIZE {world}"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    from nano_gpic_b200.config.ladder import SIZES, train_flops_per_image
    s = SIZES[a.size]
    T = a.caption_len
    if a.impl == "reference":
        res, why = run_reference(a, rank, world, dev)
        if res is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
            return
        ms, e2e_ms, launches, clocks, _ = res
    else:
        ms, e2e_ms, launches, clocks, _ = run_ours(a, rank, world, dev)
    ms = max_over_ranks(ms, dev)
    e2e_ms = max_over_ranks(e2e_ms, dev) if e2e_ms is not None else None
    peak_gb = max_over_ranks(torch.cuda.max_memory_allocated(dev) / 2 ** 30, dev) if dev.type == "cuda" else None
    pk, pk_src = peaks()
    value = a.global_batch / (ms / 1000.0)
    flops_img = train_flops_per_image(s, T)
    mfu = value * flops_img / (world * pk)
    B = a.global_batch // world
    if rank == 0:
        rec = {"metric": "train images/sec/box + MFU at d12/d18 (256px, bs1024)", "value": round(value, 1),
               "unit": "images/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 2),
               "higher_is_better": True, "scaling": "strong",
               "vs_baseline": round(value / PUBLISHED[a.size], 4) if a.size in PUBLISHED else None,
               "dtype": "bf16" if a.fp8 == "none" or a.impl == "reference" else
                        ("bf16 + MXFP8 forward GEMMs (image-block qkv_x/proj/w12/w3)" if a.fp8 == "mx" else
                         "bf16 + MXFP8 forward GEMMs (image-block qkv_x/proj/w12/w3) + MXFP8 MLP dgrads (w3, w12)"),
               "data": "synthetic (uint8 images uniform, N(0,1) caption features, random-length "
                                         "masks; random-init weights)",
               "mfu": round(mfu, 4), "mfu_peak": f"{pk / 1e12:.1f} TFLOP/s bf16 ({pk_src})",
               "model_tflops_per_gpu": round(value * flops_img / world / 1e12, 1),
               "config": {"model": f"JiT-T2I {a.size} (width {s.width}, {s.image_layers} image + {s.text_layers} text "
                                   f"layers, {s.heads} heads x 64)", "global_batch": a.global_batch,
                          "seq_len": 256 + T, "image_tokens": 256, "caption_tokens": T,
                          "micro_batch": a.micro_batch or s.micro_batch, "parallelism": f"dp{world}",
                          "optimizer": "Muon (split, NS5 bf16) + AdamW, clip 1.0, WarmupFlatCooldown",
                          "recompute": a.recompute if a.impl == "ours" else "none",
                          "l2": "inputs larger than L2 (1.3 GB of step inputs per rank, activations >> 126 MB)"},
               "clocks": clocks,
               "e2e": {"value": round(a.global_batch / (e2e_ms / 1000.0), 1) if e2e_ms else None, "unit": "images/s",
                       "h2d_bytes_per_step": B * (256 * 256 * 3 + T * 2048 * 2 + T),
                       "d2h_bytes_per_step": 4} if e2e_ms else None,
               "gpu_launches": launches,
               "peak_mem_gib": round(peak_gb, 1) if peak_gb is not None else None}
        # how the data parallelism is carried out, apart from `parallelism` (which names the work: N data-parallel
        # ranks over one global batch, the same for both arms)
        if a.impl == "reference":
            fsdp = reference_uses_fsdp(a.size, world)
            rec["dp_mode"] = "fsdp2" if fsdp else "ddp"
            rec["impl"] = "reference"
            rec.pop("gpu_launches")
            rec["reference_path"] = ("baseline/_ref (unmodified copy); autocast bf16; SDPA; " +
                                     ("FSDP2 per block (fsdp_setup.shard, blocks compiled), ShardMuonAdamW, NoSync"
                                      if fsdp else "torch.compile + DDP"))
        else:
            rec["dp_mode"] = (a.dp if a.dp == "ddp" else "zero") + ("-p2p" if a.transport == "p2p" and world > 1
                                                                    else "")
        print(json.dumps(rec), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
