"""The training step: gradient accumulation over micro-batches, data-parallel gradient reduction, global-norm clip,
Muon/AdamW update, LR schedule and the bf16 weight refresh, with no host synchronisation inside a step.

This is the part of the reference's Lightning loop that runs per optimizer step
(baselines/PixelGen/src/lightning_model_gpic.py:147-174 clip, :287-350 training_step; Lightning's automatic
optimisation with accumulate_grad_batches and DDP/FSDP2 strategies), as one plain Python object.

    tr = Trainer.for_ladder("d12", world=dist_world, rank=rank)      # model, optimizer, schedule of the ladder size
    loss = tr.train_step(images_u8, captions, caption_mask)          # one optimizer step over this rank's images
"""
import math
import os

import torch
import torch.distributed as dist

from ..config.ladder import GLOBAL_BATCH, SIZES
from ..diffusion.flow_matching import JiTTrainer
from ..models.jit_t2i import JiT_T2I
from ..optim.lr_scheduler import WarmupFlatCooldown
from ..optim.muon import MuonAdamW, tag_muon_params


def uint8_to_float(img):
    """uint8 HWC [B, H, W, 3] -> fp32 CHW in [-1, 1]: ToTensor then Normalize(0.5, 0.5), as the reference's lever D
    (baselines/PixelGen/src/data/dataset/gpic_dataset.py:869-881). On CUDA one pass of csrc/elementwise.cu's
    u8_to_unit (the same fp32 arithmetic); the PyTorch form otherwise."""
    if img.is_cuda and img.is_contiguous() and img.dim() == 4 and img.shape[3] == 3 and img.shape[2] % 8 == 0:
        from .._ext import ext
        out = torch.empty(img.shape[0], 3, img.shape[1], img.shape[2], device=img.device, dtype=torch.float32)
        ext().u8_to_unit(img, out)
        return out
    return (((img.permute(0, 3, 1, 2).float() / 255.0) - 0.5) / 0.5).contiguous()


# NVTX ranges around each micro-batch's forward+backward and around the optimizer step, for nsys / ncu range filters;
# off unless NG_NVTX=1 (a range costs a host call per push/pop).
_NVTX = os.environ.get("NG_NVTX", "0") == "1"


def _nvtx_push(name):
    if _NVTX:
        torch.cuda.nvtx.range_push(name)


def _nvtx_pop():
    if _NVTX:
        torch.cuda.nvtx.range_pop()


class Trainer:
    def __init__(self, model, optimizer, scheduler=None, objective=None, accum=1, clip=1.0, flat=None, dp=None,
                 pack=None):
        self.model = model
        # packed captions (the reference's lever E, GPIC_MFU_PACK=1; off by default there too): every micro-batch's
        # caption tokens back to back, so the text blocks skip the padding
        self.pack = (os.environ.get("GPIC_MFU_PACK") == "1") if pack is None else bool(pack)
        self.opt = optimizer
        self.sched = scheduler
        self.obj = objective or JiTTrainer()
        self.accum = accum
        self.clip = clip
        self.flat = flat
        self.dp = dp  # nano_gpic_b200.parallel.ddp.DataParallel (ddp or zero mode), or None
        self.world = dp.world if dp is not None else 1
        if dp is not None and dp.owned is not None:
            optimizer.owned = dp.owned
            dp.attach_optimizer(optimizer)  # peer-memory transport: fused update + weight broadcast
        self.global_step = 0
        self.copy_stream = None
        self.last_grad_norm = None  # device scalar: the pre-clip global norm of the last step
        self.last_per_sample = None  # device [images of the step]: per-sample losses of the last step
        self.encode = None  # optional autoencoder encode applied to the float images (PixelAE with scale/shift)

    # --------------------------------------------------------------------------------------------- construction
    @classmethod
    def for_ladder(cls, size="d12", device="cuda", world=1, rank=0, micro_batch=None, global_batch=GLOBAL_BATCH,
                   max_steps=None, dp="ddp", seed=0, model_kwargs=None, bucket_mb=1000, overlap=True,
                   transport="nccl", fp8=None, recompute=None):
        """dp: "ddp" (all-reduce, as the reference's DDP sizes) or "zero" (reduce-scatter to owners, sharded
        optimizer state; the role of the reference's FSDP2 sizes). transport (zero mode): "nccl" or "p2p" (this
        package's peer-memory kernels). fp8: None (bf16), "mx" (MXFP8 forward GEMMs in the image blocks) or "mx2" (also the MLP dgrads). recompute:
        None, "image" or "all" (activation checkpointing of those blocks)."""
        s = SIZES[size]
        torch.manual_seed(seed)
        kw = s.model_kwargs()
        kw.update(model_kwargs or {})
        if fp8 is not None:
            kw["fp8"] = fp8
        if recompute is not None:
            kw["recompute"] = recompute
        model = JiT_T2I(**kw).to(device)
        tag_muon_params(model)
        from ..parallel.ddp import make_data_parallel
        _, flat, reducer = make_data_parallel(model, world, mode="ddp" if dp == "nccl" else dp, bucket_mb=bucket_mb,
                                              device=device, overlap=overlap, transport=transport)
        mb = micro_batch or s.micro_batch
        per_rank = global_batch // world
        assert per_rank % mb == 0, (global_batch, world, mb)
        opt = MuonAdamW([{"params": [p for p in model.parameters() if p.requires_grad]}], lr=s.adamw_lr,
                        betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, muon_lr=s.muon_lr, muon_weight_decay=s.muon_wd,
                        muon_momentum=0.95, muon_nesterov=True, ns_steps=5, split=True, fused_adamw=True,
                        ns_dtype="bfloat16", update_scale="mup")
        steps = max_steps or s.steps
        wu, cd = s.schedule()
        sched = WarmupFlatCooldown(wu, cd, steps, min_lr=3e-5)(opt)
        if reducer is not None:
            reducer.broadcast_params(0)
        return cls(model, opt, sched, JiTTrainer(), accum=per_rank // mb, clip=1.0, flat=flat, dp=reducer)

    # --------------------------------------------------------------------------------------------------- step
    def _to_device(self, t, dev):
        if t.device == dev:
            return t
        return t.to(dev, non_blocking=True)

    def _stage(self, mbatch, dev):
        """(images, captions, mask, t, noise) of one micro-batch on the device. Host tensors (pinned) are copied on a
        side stream that the compute stream then waits for, so the copies of micro-batch i + 1 overlap the compute of
        micro-batch i."""
        items = [mbatch[k] if len(mbatch) > k else None for k in range(5)]
        host = dev.type == "cuda" and any(t is not None and t.device.type == "cpu" for t in items)
        if not host:
            return tuple(self._to_device(t, dev) if t is not None else None for t in items), None
        if self.copy_stream is None:
            self.copy_stream = torch.cuda.Stream(device=dev)
        cur = torch.cuda.current_stream(dev)
        with torch.cuda.stream(self.copy_stream):  # fresh device memory, pinned host sources: nothing to wait for
            out = tuple(t.to(dev, non_blocking=True) if t is not None else None for t in items)
            ready = torch.cuda.Event()
            ready.record(self.copy_stream)
        for t in out:
            if t is not None:
                t.record_stream(cur)  # freed only after the compute stream's uses
        return out, ready

    def _split(self, images, captions, caption_mask=None, t=None, noise=None):
        B = images.shape[0]
        assert B % self.accum == 0
        mb = B // self.accum
        micros = []
        for i in range(self.accum):
            sl = slice(i * mb, (i + 1) * mb)
            micros.append((images[sl], captions[sl], caption_mask[sl] if caption_mask is not None else None,
                           t[sl] if t is not None else None, noise[sl] if noise is not None else None))
        return micros

    @staticmethod
    def _key(mbatch):
        return tuple((x.data_ptr(), tuple(x.shape), x.dtype) if x is not None else None for x in mbatch)

    def train_step(self, images, captions, caption_mask=None, t=None, noise=None):
        """One optimizer step over this rank's batch, split into `accum` micro-batches.
        images: uint8 [B, H, W, 3] or float [B, 3, H, W] in [-1, 1] (host pinned or device);
        captions [B, T, D] (bf16); caption_mask [B, T] bool or None. Returns the batch-mean loss (device scalar)."""
        return self.train_micro(self._split(images, captions, caption_mask, t, noise))

    def prefetch_micro(self, mbatch):
        """prefetch() for a list-of-micro-batches caller (train_micro): stages one micro-batch (images, captions,
        mask[, t, noise]) now; the next train_micro whose first micro-batch is these tensors uses the staged copy."""
        dev = self.flat.data.device if self.flat is not None else next(self.model.parameters()).device
        self._prefetched = (self._key(tuple(mbatch)), self._stage(tuple(mbatch), dev))

    def prefetch(self, images, captions, caption_mask=None, t=None, noise=None):
        """Starts the host -> device copies of a later step's first micro-batch now (same arguments as train_step),
        on the copy stream: called right after train_step, they overlap the step the GPU is still running, so the next
        train_step with these tensors does not wait for its first copy. Host tensors only (device ones need no copy)."""
        first = self._split(images, captions, caption_mask, t, noise)[0]
        dev = self.flat.data.device if self.flat is not None else next(self.model.parameters()).device
        self._prefetched = (self._key(first), self._stage(first, dev))

    def train_micro(self, micros):
        """One optimizer step over a list of micro-batches (images, captions, mask[, t, noise]); the micro-batches may
        have different caption lengths T (length-grouped or bucketed loaders). Gradients are the mean over all images
        of all micro-batches of all ranks (micro-batches of equal size)."""
        dev = self.flat.data.device if self.flat is not None else next(self.model.parameters()).device
        if self.flat is not None:
            self.flat.zero_grad()
        n = len(micros)
        losses = []
        # caption lengths on the host for packing, read from the loader's host masks before the copies
        host_lens = [(mc[2].sum(1).tolist() if mc[2] is not None and mc[2].device.type == "cpu" else None)
                     for mc in micros] if self.pack else [None] * n
        pre = getattr(self, "_prefetched", None)
        self._prefetched = None
        staged = pre[1] if pre is not None and pre[0] == self._key(tuple(micros[0])) else self._stage(micros[0], dev)
        for i in range(n):
            (x, y, m, ti, ni), ready = staged
            if ready is not None:  # this micro-batch's copies, enqueued one micro-batch earlier
                torch.cuda.current_stream(dev).wait_event(ready)
            if i + 1 < n:  # the next micro-batch's host -> device copies run on a side stream under this one's compute
                staged = self._stage(micros[i + 1], dev)
            if self.dp is not None and i == n - 1:
                self.dp.arm()
            x = uint8_to_float(x) if x.dtype == torch.uint8 else x.float()
            if self.encode is not None:
                x = self.encode(x)
            y = y.to(torch.bfloat16)
            y_pack = None
            if self.pack:
                from ..parallel.rebalance import pack_captions
                if m is None:
                    m = torch.ones(y.shape[:2], dtype=torch.bool, device=y.device)
                y, y_pack = pack_captions(y, m, host_lens[i])
                m = None
            # mean over this rank's images and over ranks (the collectives sum)
            _nvtx_push(f"micro {i} fwd+bwd")
            per = self.obj.train_step(self.model, x, y, m, t=ti, noise=ni,
                                      grad_scale=1.0 / (x.numel() * n * self.world),
                                      **({"y_pack": y_pack} if y_pack is not None else {}))
            _nvtx_pop()
            losses.append(per)
        _nvtx_push("optimizer")
        if self.dp is not None:
            self.dp.finish_grads()
        self.last_grad_norm = self.clip_grad()
        self.opt.step()
        if self.sched is not None:
            self.sched.step()
        if self.dp is not None:
            self.dp.refresh_weights()
        elif self.flat is not None:
            self.flat.sync_bf16()
        if hasattr(self.model, "weights_changed"):
            self.model.weights_changed()
        _nvtx_pop()
        self.global_step += 1
        self.last_per_sample = torch.cat(losses)  # per-sample losses of the step, micro-batch order (device)
        return self.last_per_sample.mean()

    @torch.no_grad()
    def clip_grad(self):
        """Global 2-norm clip (max_norm = self.clip), on the device: coef = min(1, max / (norm + 1e-6))."""
        if not self.clip:
            return None
        if self.dp is not None:
            norm = self.dp.grad_norm()
            self.dp.scale_grads((self.clip / (norm + 1e-6)).clamp(max=1.0))
            return norm
        if self.flat is not None:
            norm = self.flat.grad.norm()
            from ..ops.optim import scale_
            scale_(self.flat.grad, (self.clip / (norm + 1e-6)).clamp(max=1.0))
            return norm
        return torch.nn.utils.clip_grad_norm_([p for p in self.model.parameters() if p.grad is not None], self.clip)
