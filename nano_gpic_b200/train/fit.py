"""`main.py fit` and `main.py predict`: build everything a composed configuration names and run it.

fit (the reference's LightningCLI fit: baselines/PixelGen/main.py, src/lightning_model_gpic.py:48-430,
src/lightning_data_gpic.py:51-147) on every rank of a torchrun launch:
    distributed init (NCCL on GPUs, gloo otherwise; rendezvous from the environment)
    denoiser, pixel autoencoder, conditioner, objective from model.*; Muon tags when the optimizer is MuonAdamW
    flat layout + data parallelism (trainer.strategy: DDP -> "ddp", FSDP -> "zero"; bucket_cap_mb)
    optimizer, LR schedule, EMA (model.ema_tracker; off with GPIC_MFU_NO_EMA=1: checkpoints mirror the raw weights)
    callbacks (trainer.callbacks), run directory <default_root_dir>/exp_<tags.exp>, the resolved config written there
    resume from ckpt_path ("last" = the newest last*.ckpt of the run directory)
    the loop: accumulate_grad_batches micro-batches of data.train_batch_size per optimizer step, until max_steps
    or a SIGTERM stop; logs every trainer.log_every_n_steps steps (loss, lr, images/s, per-caption-type losses) to
    metrics.jsonl and, when the trainer's logger node names a W&B logger, to an offline W&B run (train/metrics.py);
    log steps are the only host synchronisations.
predict: sampling with model.diffusion_sampler over data.pred_dataset prompts, images written by SaveImagesHook.

GPIC_SYNTHETIC=1 (or data.synthetic: true) trains on synthetic batches of the configured shape.
"""
import datetime
import json
import os
import time

import torch
import torch.distributed as dist

from ..config.cli import get_dotted, instantiate, is_spec, resolve, run_dir, strategy_mode, write_config
from ..data.pil_resize import ResizeBatch
from ..parallel.rebalance import Rebalancer
from .callbacks import EMASpec, Warmup
from .checkpoint import AsyncWriter, build_checkpoint, clean_tmp, find_resume, load_into, save_sync
from .trainer import Trainer


def init_distributed():
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if torch.cuda.is_available():
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
    else:
        dev = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        timeout = datetime.timedelta(minutes=float(os.environ.get("GPIC_PG_TIMEOUT_MIN", 30)))
        if dev.type == "cuda":
            dist.init_process_group("nccl", timeout=timeout, device_id=dev)
        else:
            dist.init_process_group("gloo", timeout=timeout)
    return rank, world, dev


class FitContext:
    def __init__(self, trainer, ema, run_dir, rank, world, device, cfg, max_steps, micro_batch, writer, callbacks):
        self.trainer, self.ema, self.run_dir = trainer, ema, run_dir
        self.rank, self.world, self.device, self.cfg = rank, world, device, cfg
        self.max_steps, self.micro_batch, self.writer, self.callbacks = max_steps, micro_batch, writer, callbacks
        self.stop = False
        self.sinks = None  # MetricSinks (metrics.jsonl, W&B when configured)

    def save(self, name, full, dirpath=None, wait=False):
        """Collective: every rank calls it (zero mode gathers the sharded state); rank 0 writes."""
        tr = self.trainer
        if tr.dp is not None:
            tr.dp.prepare_checkpoint(tr.opt, self.ema, full)
        extra = {type(c).__name__: c.state_dict() for c in self.callbacks if c.state_dict() is not None}
        ck = build_checkpoint(tr, full, self.ema, extra_callbacks=extra)
        path = os.path.join(dirpath or self.run_dir, name)
        if self.rank == 0:
            os.makedirs(os.path.dirname(path), exist_ok=True)
            if self.writer is not None:
                self.writer.save(ck, path)
                if wait:
                    self.writer.wait()
            else:
                save_sync(ck, path)
            print(f"[ckpt] step {tr.global_step} ({tr.global_step * tr.accum} micro-batches): {name}", flush=True)
        return path

    def log(self, values, step):
        if self.sinks is None:
            from .metrics import MetricSinks
            self.sinks = MetricSinks(self.run_dir, self.rank)
        self.sinks.log(values, step)


def _seed_everything(seed):
    import random
    import numpy as np
    random.seed(seed)
    np.random.seed(seed % (2 ** 32))
    torch.manual_seed(seed)


def build_model_parts(cfg, device):
    m = cfg.get("model") or {}
    den = instantiate(m["denoiser"]).to(device)
    vae = instantiate(m["vae"]) if is_spec(m.get("vae")) else None
    obj = instantiate(m["diffusion_trainer"]) if is_spec(m.get("diffusion_trainer")) else None
    cond = None
    if is_spec(m.get("conditioner")):
        node = m["conditioner"]
        cond = instantiate(node, device=device) if "Qwen3" in node["class_path"] else instantiate(node)
    return den, vae, cond, obj


def _loader(cfg, rank, world, device, den, start=0):
    """(iterator over micro-batches, micro-batch size); start = micro-batches already consumed (a resume; the real
    loader resumes through the shard clock instead)."""
    d = cfg.get("data") or {}
    mb = int(d.get("train_batch_size", 32))
    synthetic = os.environ.get("GPIC_SYNTHETIC") == "1" or d.get("synthetic") or not is_spec(d.get("train_dataset"))
    if synthetic:
        from ..data.gpic import SyntheticGPIC
        T = int(d.get("synthetic_caption_len", 128))
        return iter(SyntheticGPIC(mb, T=T, D=den.txt_embed_dim, image_size=den.input_size, seed=1000 + rank,
                                  start=start)), mb
    ds = instantiate(d["train_dataset"], batch_size=mb)
    loader = ds.build_dataloader(mb, num_workers=int(d.get("train_num_workers", 8)))
    if getattr(ds, "shared_bucket", False):
        from ..data.buckets import SharedBucketLoader
        loader = SharedBucketLoader(loader)
    return iter(loader), mb


def fit(cfg):
    rank, world, dev = init_distributed()
    _seed_everything(int(cfg.get("seed_everything") or 0))
    tcfg = cfg.get("trainer") or {}
    m = cfg.get("model") or {}
    den, vae, cond, obj = build_model_parts(cfg, dev)
    ocfg = m.get("optimizer") or {"class_path": "torch.optim.AdamW", "init_args": {"lr": 1e-4}}
    if resolve(ocfg["class_path"]).__name__ == "MuonAdamW":
        from ..optim.muon import tag_muon_params
        tag_muon_params(den)
    from ..parallel.ddp import make_data_parallel
    strat = tcfg.get("strategy")
    bucket_mb = (strat.get("init_args") or {}).get("bucket_cap_mb", 1000) if is_spec(strat) else 1000
    layout, flat, dp = make_data_parallel(den, world, mode=strategy_mode(tcfg), bucket_mb=bucket_mb, device=dev)
    opt = instantiate(ocfg, params=[{"params": [p for p in den.parameters() if p.requires_grad]}])
    sched = instantiate(m["lr_scheduler"])(opt) if is_spec(m.get("lr_scheduler")) else None
    accum = int(tcfg.get("accumulate_grad_batches") or 1)
    clip = tcfg.get("gradient_clip_val", 1.0)
    trainer = Trainer(den, opt, sched, obj, accum=accum, clip=clip or 0, flat=flat, dp=dp)
    if vae is not None and (vae.scale != 1.0 or vae.shift != 0.0):
        trainer.encode = vae.encode
    if dp is not None:
        dp.broadcast_params(0)
    ema_spec = instantiate(m["ema_tracker"]) if is_spec(m.get("ema_tracker")) else EMASpec()
    ema = ema_spec.build(flat, ranges=dp.own_ranges() if dp is not None else None)
    if dp is None or dp.p2p is None:  # the update kernels apply the EMA in the same pass (peer memory: its own kernel)
        ema.attach(opt)

    rdir = run_dir(cfg)
    if rank == 0:
        os.makedirs(rdir, exist_ok=True)
        write_config(cfg, rdir)
        stale = clean_tmp(rdir)  # partial checkpoints of writers killed with an earlier launch
        if stale:
            print(f"[ckpt] removed {stale} partial checkpoint file(s) of an earlier launch", flush=True)
    callbacks = [instantiate(c) for c in (tcfg.get("callbacks") or [])]
    max_steps = int(tcfg.get("max_steps") or get_dotted(cfg, "model.lr_scheduler.init_args.max_steps") or 1)
    writer = AsyncWriter() if rank == 0 and os.environ.get("GPIC_MFU_ASYNC_CKPT", "1") != "0" else None
    mb = int((cfg.get("data") or {}).get("train_batch_size", 32))
    ctx = FitContext(trainer, ema, rdir, rank, world, dev, cfg, max_steps, mb, writer, callbacks)
    from .metrics import MetricSinks, caption_type_losses
    ctx.sinks = MetricSinks(rdir, rank, logger_node=tcfg.get("logger"), config=cfg)
    for c in callbacks:
        c.setup(ctx)

    ck_path = cfg.get("ckpt_path")
    if ck_path in ("last", "auto"):
        ck_path = find_resume(rdir)
    if ck_path:
        ck = torch.load(ck_path, map_location="cpu", weights_only=False)
        load_into(trainer, ck, ema=ema)
        if rank == 0:
            print(f"[resume] {ck_path} at step {trainer.global_step}", flush=True)
    it, mb = _loader(cfg, rank, world, dev, den, start=trainer.global_step * accum)
    for c in callbacks:
        c.on_train_start(ctx)
    if not any(isinstance(c, Warmup) for c in callbacks) and trainer.global_step > 0:
        from .checkpoint import reseed
        reseed(int(cfg.get("seed_everything") or 0), trainer.global_step)

    log_every = int(tcfg.get("log_every_n_steps") or 100)
    # sample rebalancing over ranks by caption length (reference levers E / E2): trainer.rebalance or
    # GPIC_MFU_REBALANCE = 1 (device exchange) or 2 (host exchange before the copy)
    rebal_mode = int(get_dotted(cfg, "trainer.rebalance", os.environ.get("GPIC_MFU_REBALANCE", "0")) or 0)
    rebal = Rebalancer() if rebal_mode and dist.is_initialized() and dist.get_world_size() > 1 else None
    t_log, n_log = time.perf_counter(), 0
    def fetch_micro():
        img, caps, meta = next(it)
        mtypes = list(meta.get("caption_type") or [])
        if isinstance(img, ResizeBatch):  # the bicubic crop passes of the batch, on the device
            img = img.run(dev)
        if cond is not None:
            y, uncond = cond(caps, meta)
            mask = meta.get("y_mask")
            if obj is not None and obj.null_condition_p > 0:
                y, mask = obj.caption_dropout(y.to(dev), mask, uncond.to(dev))
        else:
            y, mask = meta["text_emb"], meta["text_mask"]
        if rebal is not None and mask is not None:
            if rebal_mode == 1 or img.is_cuda:  # lever E: exchange on the device (NCCL)
                img, y, mask = img.to(dev), y.to(dev), mask.to(dev)
            img, y, mask = rebal(img, y, mask)  # host tensors (lever E2): exchange over gloo
        return (img, y, mask), mtypes

    ahead = None  # the next step's first micro-batch, fetched (and its copies started) during the previous step
    try:
        while trainer.global_step < max_steps and not ctx.stop:
            step = trainer.global_step
            micros, types = [], []
            for k in range(accum):
                mbatch, mtypes = ahead if (k == 0 and ahead is not None) else fetch_micro()
                types += mtypes
                micros.append(mbatch)
            ahead = None
            for c in callbacks:
                c.on_step_start(ctx, step)
            loss = trainer.train_micro(micros)
            ema.step(trainer.global_step)
            n_log += 1
            for c in callbacks:
                c.on_step_end(ctx, trainer.global_step, loss)
            if trainer.global_step % log_every == 0 or trainer.global_step == max_steps:
                dt = time.perf_counter() - t_log
                imgs = n_log * accum * mb * world
                vals = {"loss": float(loss), "lr": opt.param_groups[0]["lr"], "images_per_s": imgs / max(dt, 1e-9)}
                if rebal is None and trainer.last_per_sample is not None:
                    # collective (every rank, every log step); samples whose type is unknown count for no type
                    n = trainer.last_per_sample.numel()
                    vals.update(caption_type_losses(trainer.last_per_sample, types if len(types) == n else [""] * n))
                ctx.log(vals, trainer.global_step)
                if rank == 0:
                    print(f"[step {trainer.global_step}] " + " ".join(f"{k}={v:.5g}" for k, v in vals.items()),
                          flush=True)
                t_log, n_log = time.perf_counter(), 0
            # after the step's callbacks (checkpoints record the data position first): the next step's first
            # micro-batch, whose host -> device copies then run under this step's queued work
            if trainer.global_step < max_steps and not ctx.stop:
                ahead = fetch_micro()
                trainer.prefetch_micro(ahead[0])
        for c in callbacks:
            c.on_train_end(ctx)
    finally:
        if writer is not None:
            writer.close()
        if ctx.sinks is not None:
            ctx.sinks.close()
        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()
    return 0


@torch.no_grad()
def predict(cfg):
    """Samples for data.pred_dataset prompts with model.diffusion_sampler; the EMA weights of ckpt_path unless
    model.eval_original_model (reference lightning_model_gpic.py:352-373)."""
    from ..diffusion.sampling import fp2uint8
    from .callbacks import SaveImagesHook
    rank, world, dev = init_distributed()
    m, d = cfg.get("model") or {}, cfg.get("data") or {}
    den, vae, cond, _ = build_model_parts(cfg, dev)
    ck_path = cfg.get("ckpt_path")
    if ck_path:
        sd = torch.load(ck_path, map_location="cpu", weights_only=False)
        sd = sd.get("state_dict", sd)
        prefix = "denoiser." if m.get("eval_original_model") else "ema_denoiser."
        den.load_state_dict({k[len(prefix):]: v for k, v in sd.items() if k.startswith(prefix)}, strict=False)
    den.eval()
    sampler = instantiate(m["diffusion_sampler"])
    ds = instantiate(d["pred_dataset"])
    bs = int(d.get("pred_batch_size", 8))
    idx = list(range(rank, len(ds), world))
    rdir = run_dir(cfg)
    if rank == 0:
        os.makedirs(rdir, exist_ok=True)
        write_config(cfg, rdir, stage="TrainerFn.PREDICTING")
    hook = SaveImagesHook(save_dir=os.environ.get("GPIC_PRED_DIR", "predict"))
    ctx = FitContext(None, None, rdir, rank, world, dev, cfg, 0, bs, None, [])
    images, metas = [], []
    # the denoiser's forward replayed from a CUDA graph per batch shape (sampling at small batches is launch-bound);
    # GPIC_PRED_GRAPHS=0 runs it eagerly
    from ..runtime.graphs import GraphedCall
    den_call = (GraphedCall(lambda x, t, yy, mm: den(x, t, yy, y_mask=mm))
                if os.environ.get("GPIC_PRED_GRAPHS", "1") != "0" else (lambda x, t, yy, mm: den(x, t, yy, y_mask=mm)))
    for s in range(0, len(idx), bs):
        items = [ds[i] for i in idx[s:s + bs]]
        noise = torch.stack([it[0] for it in items]).to(dev)
        caps = [it[1] for it in items]
        meta = {}
        y, uncond = cond(caps, meta)
        mask = meta["y_mask"]
        null_mask = torch.zeros_like(mask)
        null_mask[:, 0] = True
        cfg_on = float(sampler.guidance) != 1.0

        def net(x, t, yy):
            mm = torch.cat([null_mask, mask]) if cfg_on and yy.shape[0] == 2 * mask.shape[0] else mask
            return den_call(x, t, yy, mm)

        x = sampler(net, noise, y, uncond)
        if vae is not None:
            x = vae.decode(x)
        u8 = fp2uint8(x).permute(0, 2, 3, 1).cpu().numpy()
        images += list(u8)
        metas += [it[2] for it in items]
    import numpy as np
    hook.write(ctx, np.stack(images) if images else np.zeros((0,)), metas)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0
