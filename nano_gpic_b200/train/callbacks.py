"""Training-loop callbacks with the reference's names and constructor arguments, so its YAML callback lists build them
(reference baselines/PixelGen/src/callbacks/*.py). A callback is a plain object with optional hooks, called by
nano_gpic_b200.train.fit on every rank:

    setup(ctx)                     once, after the model, optimizer, data parallelism and run directory exist
    on_train_start(ctx)            before the first step (after a resume's checkpoint is loaded)
    on_step_start(ctx, step)       before each optimizer step (step = the global step it will produce - 1)
    on_step_end(ctx, step, loss)   after each optimizer step, step = new global step, loss a device scalar
    on_train_end(ctx)
    state_dict() -> dict | None    stored under checkpoint["callbacks"][ClassName]

ctx is the FitContext (trainer, ema, policy, run_dir, rank, world, device, cfg, log). No hook synchronises the host
with the device except where the reference's does (log steps, checkpoint steps).
"""
import gc
import hashlib
import json
import os
import sys
import time

import torch
import torch.distributed as dist


class Callback:
    def setup(self, ctx):
        pass

    def on_train_start(self, ctx):
        pass

    def on_step_start(self, ctx, step):
        pass

    def on_step_end(self, ctx, step, loss):
        pass

    def on_train_end(self, ctx):
        pass

    def state_dict(self):
        return None


# ---------------------------------------------------------------------------------------------------- checkpoints
def lightning_name(filename, step):
    """Lightning's checkpoint file name: "ms-{step:06d}" -> "ms-step=000100.ckpt"."""
    return filename.replace("{step", "step={step").format(step=step) + ".ckpt"


class CheckpointHook(Callback):
    """Every `every_n_train_steps` steps: `filename` (model and EMA weights only, as the reference strips optimizer,
    loops and callbacks from non-last files) when save_top_k != 0, and `last.ckpt` (full state) when save_last.
    Never at the step the launch resumed from; also at max_steps for the ms files (reference
    src/callbacks/model_checkpoint.py:9-69)."""

    def __init__(self, filename="ms-{step:06d}", every_n_train_steps=0, save_last=False, save_top_k=-1, monitor=None,
                 dirpath=None):
        self.filename, self.every = filename, int(every_n_train_steps or 0)
        self.save_last, self.save_files = bool(save_last), save_top_k != 0
        self.dirpath = dirpath
        self.resumed = None

    def on_train_start(self, ctx):
        self.resumed = ctx.trainer.global_step

    def on_step_end(self, ctx, step, loss):
        if step == self.resumed:
            return
        at_every = self.every and step % self.every == 0
        if self.save_files and (at_every or step == ctx.max_steps):
            ctx.save(lightning_name(self.filename, step), full=False, dirpath=self.dirpath)
        if self.save_last and at_every:
            ctx.save("last.ckpt", full=True, dirpath=self.dirpath)


class SaveOnTermCallback(Callback):
    """SIGTERM sets a flag; every `every` steps one MAX all-reduce decides a common step at which all ranks save
    last-term.ckpt and stop (reference src/callbacks/save_on_term.py:21-56)."""

    def __init__(self, every=20, filename="last-term.ckpt"):
        from .checkpoint import SaveOnTerm
        self.impl = SaveOnTerm(every=every, filename=filename)

    def on_step_end(self, ctx, step, loss):
        if self.impl.check(step, device=ctx.device):
            ctx.save(self.impl.filename, full=True, wait=True)
            ctx.stop = True


class ShardClock(Callback):
    """The data-shard clock {time, seed, step} stored in every checkpoint under `gpic_shard_clock` (the checkpoint
    builder writes it); this callback takes the shard seed from <run_dir>/shard_seed.txt when the environment has none
    (reference src/callbacks/shard_clock.py:18-20, jobs/final_ladder.sh:39)."""

    def setup(self, ctx):
        path = os.path.join(ctx.run_dir, "shard_seed.txt")
        if "GPIC_SHARD_SEED" not in os.environ and os.path.exists(path):
            with open(path) as f:
                os.environ["GPIC_SHARD_SEED"] = f.read().strip()


# --------------------------------------------------------------------------------------------------- warm-up
def _progress(ctx):
    """Rank 0 touches <GPIC_FIRST_STEP_FILE>.progress: start-up work is still advancing (launch_guard.py)."""
    path = os.environ.get("GPIC_FIRST_STEP_FILE")
    if path and ctx.rank == 0:
        with open(path + ".progress", "a"):
            os.utime(path + ".progress", None)


class Warmup(Callback):
    """Before the first step, the real forward + backward on dummy batches at caption lengths T (64, 128, 320, 192 by
    default) on every rank, then the gradients are zeroed and the weights are untouched: kernels' tensor maps,
    function attributes, workspaces and the allocator's pools exist before timing starts (the reference compiles its
    graphs here, src/callbacks/compile_warmup.py:19-90). On a resume every RNG is reseeded from
    (seed * 1000003 + step) so a resumed launch draws the same numbers."""

    def __init__(self, lengths=(64, 128, 320, 192), micro_batch=None, seed=0):
        self.lengths, self.micro_batch, self.seed = tuple(lengths), micro_batch, seed

    def on_train_start(self, ctx):
        tr = ctx.trainer
        model = tr.model
        dev = ctx.device
        B = self.micro_batch or ctx.micro_batch
        D = getattr(model, "txt_embed_dim", 2048)
        size = getattr(model, "input_size", 256)
        cin = getattr(model, "in_channels", 3)
        g = torch.Generator().manual_seed(1234)
        for T in self.lengths:
            T = min(T, getattr(model, "txt_max_length", T))
            x = (torch.rand(B, cin, size, size, generator=g) * 2 - 1).to(dev)
            y = torch.randn(B, T, D, generator=g).to(dev, torch.bfloat16)
            m = torch.ones(B, T, dtype=torch.bool, device=dev)
            tr.obj.train_step(model, x, y, m, grad_scale=1.0 / x.numel())
            _progress(ctx)  # the launch watchdog restarts its clock at each finished warm-up length
        if tr.flat is not None:
            tr.flat.zero_grad()
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        if tr.global_step > 0:
            from .checkpoint import reseed
            reseed(self.seed, tr.global_step)


class HostTuning(Callback):
    """Host placement of a rank (reference src/callbacks/host_tuning.py:16-140): bind the process to the CPUs of its
    GPU's NUMA node, freeze the garbage collector's current objects after warm-up (fewer full collections in the hot
    loop), and optionally seed Python/NumPy per rank."""

    def __init__(self, numa=True, gc_freeze=True, seed_per_rank=False):
        self.numa, self.gc_freeze, self.seed_per_rank = numa, gc_freeze, seed_per_rank
        self.cpus = None

    @staticmethod
    def gpu_cpus(device_index):
        """CPU ids of the NUMA node of a GPU, from sysfs (empty when unknown)."""
        try:
            bus = torch.cuda.get_device_properties(device_index).pci_bus_id if hasattr(
                torch.cuda.get_device_properties(device_index), "pci_bus_id") else None
        except Exception:
            bus = None
        if not bus:
            return []
        bus = bus.lower()
        if len(bus.split(":")[0]) > 4:
            bus = bus[len(bus.split(":")[0]) - 4:]
        try:
            with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
                node = int(f.read())
            if node < 0:
                return []
            with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
                return parse_cpulist(f.read())
        except OSError:
            return []

    def setup(self, ctx):
        if self.numa and ctx.device.type == "cuda":
            cpus = self.gpu_cpus(ctx.device.index)
            if cpus:
                os.sched_setaffinity(0, cpus)
                self.cpus = cpus
        if self.seed_per_rank:
            import random
            import numpy as np
            random.seed(ctx.rank)
            np.random.seed(ctx.rank)

    def on_train_start(self, ctx):
        if self.gc_freeze:
            gc.collect()
            gc.freeze()


def parse_cpulist(text):
    out = []
    for part in text.strip().split(","):
        if not part:
            continue
        a, _, b = part.partition("-")
        out += list(range(int(a), int(b or a) + 1))
    return out


class FirstStepMarker(Callback):
    """Rank 0 writes the file named by GPIC_FIRST_STEP_FILE after the first step (the launch watchdog's signal that
    training started; reference src/callbacks/first_step.py:14-31)."""

    def __init__(self, path=None):
        self.path = path or os.environ.get("GPIC_FIRST_STEP_FILE")
        self.done = False

    def on_step_end(self, ctx, step, loss):
        if self.done or not self.path or ctx.rank != 0:
            return
        self.done = True
        os.makedirs(os.path.dirname(os.path.abspath(self.path)), exist_ok=True)
        with open(self.path, "w") as f:
            f.write(f"{step} {time.time():.3f}\n")


# --------------------------------------------------------------------------------------------------- measurement
class BenchTimer(Callback):
    """Per-step timing without syncing the host every step (reference src/callbacks/bench.py:1-250): CUDA events
    around each optimizer step give the GPU span; wall clock gives the step-to-step time and the host time spent
    before the step's work was queued; memory peaks. Events are read `lag` steps later, so only the log step
    waits. Records go to <run_dir>/bench.jsonl (rank 0) every `every` steps; `profile_steps=(a, b)` runs
    torch.profiler over steps [a, b) and writes a Chrome trace."""

    def __init__(self, every=50, lag=2, profile_steps=None, filename="bench.jsonl"):
        self.every, self.lag, self.profile_steps, self.filename = every, lag, profile_steps, filename
        self.pending, self.rows = [], []
        self.t_prev = None
        self.prof = None

    def on_step_start(self, ctx, step):
        self.t0 = time.perf_counter()
        if ctx.device.type == "cuda":
            self.ev0 = torch.cuda.Event(enable_timing=True)
            self.ev0.record()
        if self.profile_steps and step == self.profile_steps[0]:
            self.prof = torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU,
                                                           torch.profiler.ProfilerActivity.CUDA])
            self.prof.__enter__()

    def on_step_end(self, ctx, step, loss):
        t1 = time.perf_counter()
        row = {"step": step, "host_ms": (t1 - self.t0) * 1e3,
               "step_to_step_ms": (t1 - self.t_prev) * 1e3 if self.t_prev else None}
        self.t_prev = t1
        if ctx.device.type == "cuda":
            ev1 = torch.cuda.Event(enable_timing=True)
            ev1.record()
            self.pending.append((row, self.ev0, ev1))
        else:
            self.rows.append(row)
        if self.prof is not None and step + 1 >= self.profile_steps[1]:
            self.prof.__exit__(None, None, None)
            if ctx.rank == 0:
                self.prof.export_chrome_trace(os.path.join(ctx.run_dir, f"trace_steps{self.profile_steps[0]}.json"))
            self.prof = None
        if step % self.every == 0:
            self.flush(ctx)

    def flush(self, ctx):
        if self.pending:
            self.pending[-1][2].synchronize()
            for row, a, b in self.pending:
                row["gpu_ms"] = a.elapsed_time(b)
                self.rows.append(row)
            self.pending = []
            row = self.rows[-1]
            row["max_mem_gb"] = torch.cuda.max_memory_allocated(ctx.device) / 2 ** 30
        if ctx.rank == 0 and self.rows:
            with open(os.path.join(ctx.run_dir, self.filename), "a") as f:
                for r in self.rows:
                    f.write(json.dumps(r) + "\n")
        self.rows = []

    def on_train_end(self, ctx):
        self.flush(ctx)


def _digest(tensors):
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.detach().float().contiguous().cpu().numpy().tobytes())
    return h.hexdigest()[:16]


class LaunchFingerprint(Callback):
    """Hashes of the parameters, the optimizer state and the RNG states at the first step of a launch, written to
    <run_dir>/fingerprint_rank<r>.json: two launches (e.g. a resume and an uninterrupted run) can be compared
    (reference src/callbacks/launch_fingerprint.py:1-175)."""

    def __init__(self, filename="fingerprint_rank{rank}.json"):
        self.filename = filename
        self.done = False

    def fingerprint(self, ctx):
        tr = ctx.trainer
        params = [p for p in tr.model.parameters()]
        state = []
        for st in tr.opt.state.values():
            state += [v for v in st.values() if torch.is_tensor(v)]
        rng = [torch.get_rng_state()]
        if torch.cuda.is_available() and ctx.device.type == "cuda":
            rng.append(torch.cuda.get_rng_state(ctx.device))
        return {"step": tr.global_step, "params": _digest(params), "optimizer": _digest(state) if state else None,
                "rng": _digest([r.to(torch.uint8) for r in rng])}

    def on_step_start(self, ctx, step):
        if self.done:
            return
        self.done = True
        fp = self.fingerprint(ctx)
        with open(os.path.join(ctx.run_dir, self.filename.format(rank=ctx.rank)), "w") as f:
            json.dump(fp, f)


class NoneRefcount(Callback):
    """Logs sys.getrefcount(None) every `every` steps to <run_dir>/none_refcount.txt (rank 0). The reference guards a
    torch 2.7.1 C++-wrapper reference leak this way (src/callbacks/none_refcount.py:12-23); here it is a cheap
    leak monitor of the Python side."""

    def __init__(self, every=1000):
        self.every = every

    def on_step_end(self, ctx, step, loss):
        if ctx.rank == 0 and step % self.every == 0:
            with open(os.path.join(ctx.run_dir, "none_refcount.txt"), "a") as f:
                f.write(f"{step} {sys.getrefcount(None)}\n")


class GradientMonitor(Callback):
    """The global gradient norm (the clip's pre-clip value) logged every `every` steps (reference
    src/callbacks/grad.py:6-21)."""

    def __init__(self, every=100):
        self.every = every

    def on_step_end(self, ctx, step, loss):
        if step % self.every == 0 and ctx.trainer.last_grad_norm is not None:
            ctx.log({"grad_norm": float(ctx.trainer.last_grad_norm)}, step)


class SaveImagesHook(Callback):
    """Prediction: every rank's uint8 samples gathered to rank 0 and written to <run_dir>/<save_dir>/output.npz, plus
    one PNG per sample through each sample's save_fn (reference src/callbacks/save_images.py:16-115)."""

    def __init__(self, save_dir="val", save_compressed=False):
        self.save_dir, self.save_compressed = save_dir, save_compressed

    def write(self, ctx, images, metas):
        import numpy as np
        root = os.path.join(ctx.run_dir, self.save_dir)
        os.makedirs(root, exist_ok=True)
        for img, meta in zip(images, metas):
            fn = meta.get("save_fn")
            if fn is not None:
                fn(img, meta, root)
        allimg = [images]
        if ctx.world > 1:
            allimg = [None] * ctx.world
            dist.all_gather_object(allimg, images)
        if ctx.rank == 0:
            arr = np.concatenate([a for a in allimg if len(a)], 0) if any(len(a) for a in allimg) else np.zeros(0)
            (np.savez_compressed if self.save_compressed else np.savez)(os.path.join(root, "output.npz"), arr_0=arr)


class EMASpec:
    """The `model.ema_tracker` node (reference src/callbacks/simple_ema.py init args); fit builds the SimpleEMA over
    the flat buffers from it."""

    def __init__(self, decay=0.9999, every_n_steps=1):
        self.decay, self.every_n_steps = decay, every_n_steps

    def build(self, flat, ranges=None):
        from .ema import SimpleEMA
        return SimpleEMA(flat, decay=self.decay, every_n_steps=self.every_n_steps, ranges=ranges)
