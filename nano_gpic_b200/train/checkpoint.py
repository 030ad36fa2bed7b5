"""Checkpoints in the reference's Lightning `.ckpt` layout, written off the training path.

Layout (a torch.save'd dict; reference baselines/PixelGen/src/lightning_model_gpic.py:408-430,
src/callbacks/model_checkpoint.py:9-69, src/callbacks/shard_clock.py:18-20):
    state_dict           denoiser.<param>, ema_denoiser.<param> (the EMA, or the raw weights when the run keeps no EMA)
    global_step, epoch, pytorch-lightning_version
    gpic_shard_clock     {time, seed, step}: the moment the state was taken (resume cuts the shard log there)
    full files only:     optimizer_states [optimizer.state_dict()], lr_schedulers [scheduler.state_dict()],
                         loops, callbacks (EMA state, trainer counters)
File names: ms-step=NNNNNN.ckpt (model only), last.ckpt (full state), last-term.ckpt (full state, saved on SIGTERM).
The reference's tools (heldout_loss.build_denoiser: strict load of denoiser.* / ema_denoiser.*, global_step) read these
files, and this module loads the reference's own checkpoints.

AsyncWriter has the role of the reference's AsyncShmCheckpointIO (src/plugins/async_ckpt_io.py:1-261): training
continues while a checkpoint is written. Here the training process copies the tensors into shared-memory files (one
device-to-host copy) and a writer process, fed over a pipe, writes the dict to `<file>.part-<pid>`, fsyncs it and
renames it into place (atomic), with the file's mtime set to the snapshot time. EMA twins (ema_denoiser.X bit-equal to
denoiser.X) share one storage in the file.
"""
import glob
import math
import os
import re
import signal
import tempfile
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SHARD_CLOCK_KEY = "gpic_shard_clock"
PL_VERSION = "2.6.0"
MS_NAME = "ms-step={step:06d}.ckpt"


# ----------------------------------------------------------------------------------------------------------- format
def model_state(model, prefix):
    return {prefix + k: v.detach() for k, v in model.state_dict().items()}


def build_checkpoint(trainer, full, ema=None, extra_callbacks=None):
    """The checkpoint dict of a nano_gpic_b200 Trainer (tensors still on their devices)."""
    sd = model_state(trainer.model, "denoiser.")
    if ema is not None and not ema.off:
        sd.update(ema.state_tensors("ema_denoiser."))
    else:  # no EMA: the EMA slot holds the raw weights (reference SimpleEMA.mirror)
        sd.update({"ema_denoiser." + k[len("denoiser."):]: v for k, v in list(sd.items())})
    ck = {"epoch": 0, "global_step": int(trainer.global_step), "pytorch-lightning_version": PL_VERSION,
          "state_dict": sd,
          SHARD_CLOCK_KEY: {"time": time.time(), "seed": os.environ.get("GPIC_SHARD_SEED"),
                            "step": int(trainer.global_step)}}
    if full:
        ck["optimizer_states"] = [trainer.opt.state_dict()]
        ck["lr_schedulers"] = [trainer.sched.state_dict()] if trainer.sched is not None else []
        ck["loops"] = {"fit_loop": {"epoch_loop.batch_progress": {"total": {"processed": int(trainer.global_step) *
                                                                            int(trainer.accum)}}}}
        cb = {"Trainer": {"global_step": int(trainer.global_step), "accum": int(trainer.accum)}}
        if ema is not None:
            cb["SimpleEMA"] = ema.state_dict()
        cb.update(extra_callbacks or {})
        ck["callbacks"] = cb
    return ck


def load_into(trainer, ck, strict=True, load_optimizer=True, ema=None):
    """Restore a checkpoint dict into a Trainer: the denoiser weights (strict), the EMA, the optimizer and schedule
    state when present, the global step. A pos_embed of another shape is dropped (reference
    lightning_model_gpic.py:264-285)."""
    sd = ck["state_dict"] if "state_dict" in ck else ck
    den = {k[len("denoiser."):]: v for k, v in sd.items() if k.startswith("denoiser.")}
    own = trainer.model.state_dict()
    if "pos_embed" in den and "pos_embed" in own and den["pos_embed"].shape != own["pos_embed"].shape:
        den.pop("pos_embed")
        strict = False
    trainer.model.load_state_dict(den, strict=strict)
    if ema is not None:
        e = {k[len("ema_denoiser."):]: v for k, v in sd.items() if k.startswith("ema_denoiser.")}
        if e:
            ema.load_tensors(e)
    if getattr(trainer, "flat", None) is not None:
        trainer.flat.sync_bf16()
    if hasattr(trainer.model, "weights_changed"):
        trainer.model.weights_changed()
    if load_optimizer and ck.get("optimizer_states"):
        trainer.opt.load_state_dict(ck["optimizer_states"][0])
        for st in trainer.opt.state.values():  # Lightning restores the state on the CPU; the fused AdamW wants it here
            for k, v in list(st.items()):
                if torch.is_tensor(v):
                    p_dev = trainer.flat.data.device if getattr(trainer, "flat", None) is not None else v.device
                    st[k] = v.to(p_dev)
    if load_optimizer and ck.get("optimizer_states") and getattr(trainer, "dp", None) is not None:
        trainer.dp.after_load()
    if load_optimizer and ck.get("lr_schedulers") and trainer.sched is not None:
        trainer.sched.load_state_dict(ck["lr_schedulers"][0])
    trainer.global_step = int(ck.get("global_step", 0))
    return trainer.global_step


def reseed(seed, step):
    """RNG state of a resumed run: every generator reseeded from (seed * 1000003 + step) (reference
    src/callbacks/compile_warmup.py:74-90), so a resumed run draws the same numbers at every launch."""
    s = (int(seed) * 1000003 + int(step)) % (2 ** 63)
    torch.manual_seed(s)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(s)
    return s


def find_resume(run_dir):
    """The newest last*.ckpt of a run directory (by mtime), or None (reference jobs/train_ladder.sh:79-81)."""
    c = glob.glob(os.path.join(run_dir, "last*.ckpt"))
    return max(c, key=os.path.getmtime) if c else None


def read_shard_clock(path):
    """{time, seed, step} stored in a checkpoint (reference tools/ckpt_shard_clock.py)."""
    ck = torch.load(path, map_location="cpu", mmap=True, weights_only=False)
    return ck.get(SHARD_CLOCK_KEY)


def _partial_name(path):
    """The file a checkpoint is written to before it is renamed over `path`: `<path>.part-<pid>`."""
    return f"{path}.part-{os.getpid()}"


def _publish(obj, path, stamp=None):
    """torch.save into the partial file, flush it to disk, rename it over `path` (atomic), and give the file the
    snapshot's time (the moment the state was taken, not the moment the write finished)."""
    part = _partial_name(path)
    with open(part, "wb") as f:
        torch.save(obj, f)
        f.flush()
        os.fsync(f.fileno())
    os.replace(part, path)
    if stamp is not None:
        os.utime(path, (stamp, stamp))


def save_sync(ck, path):
    """Writes a checkpoint in the calling process (tensors moved to the host first)."""
    _publish(_to_cpu(ck), path)


def _to_cpu(obj):
    return _tree_map(obj, lambda v: v.detach().cpu() if torch.is_tensor(v) else v)


def _tree_map(obj, fn):
    if isinstance(obj, dict):
        return {k: _tree_map(v, fn) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_tree_map(v, fn) for v in obj)
    return fn(obj)


# ------------------------------------------------------------------------------------------------------ async writer
# How a save travels. The training process copies every tensor of the checkpoint into a file in shared memory
# (/dev/shm; one file per slot, grown when a checkpoint needs more) and sends the writer process one message over a
# pipe: (slot, file, bytes used, skeleton, destination, snapshot time), where the skeleton is the checkpoint dict with
# each tensor replaced by a _Blob (offset, dtype, shape). The writer maps the file, turns each _Blob into a tensor
# over the mapped bytes (torch.frombuffer: no copy; one tensor per offset, so EMA twins stay one storage), writes the
# dict (_publish) and answers (slot, destination, error or None). The writer leaves when its end of the pipe reports
# EOF, which also happens when the training process dies, and removes the shared files it was given.
class _Blob:
    __slots__ = ("off", "dtype", "shape")

    def __init__(self, off, dtype, shape):
        self.off, self.dtype, self.shape = off, dtype, tuple(shape)

    def nbytes(self):
        return math.prod(self.shape) * torch.empty((), dtype=self.dtype).element_size()


def _writer_loop(conn, delay):
    import mmap
    signal.signal(signal.SIGTERM, signal.SIG_IGN)  # a TERM to the job must not cut a write short
    signal.signal(signal.SIGINT, signal.SIG_IGN)
    mapped = {}  # shared file -> (mmap, size)

    def region(name, size):
        if name not in mapped or mapped[name][1] < size:
            with open(name, "r+b") as f:
                mapped[name] = (mmap.mmap(f.fileno(), size), size)
        return mapped[name][0]

    try:
        while True:
            try:
                msg = conn.recv()
            except (EOFError, OSError):
                return
            if msg is None:
                return
            slot, shm, used, skel, dest, stamp = msg
            try:
                if delay:
                    time.sleep(delay)
                mm = region(shm, used)
                made = {}

                def tensor_of(v):
                    if not isinstance(v, _Blob):
                        return v
                    if v.off not in made:
                        n = math.prod(v.shape)
                        made[v.off] = (torch.frombuffer(mm, dtype=v.dtype, count=n, offset=v.off).view(v.shape)
                                       if n else torch.empty(v.shape, dtype=v.dtype))
                    return made[v.off]
                _publish(_tree_map(skel, tensor_of), dest, stamp)
                made.clear()
                conn.send((slot, dest, None))
            except Exception as e:  # reported in the training process at its next save or at wait()
                conn.send((slot, dest, repr(e)))
    finally:
        for name in list(mapped):
            try:
                os.unlink(name)
            except OSError:
                pass


class AsyncWriter:
    """Checkpoint writes in a separate process. `save(ck, path)` returns once the tensors are copied into shared
    memory; `wait()` blocks until every write is on disk and raises if one failed. `nbuf` slots: that many saves may
    be in flight."""

    def __init__(self, nbuf=2, delay=None):
        ctx = mp.get_context("spawn")
        self.conn, child = ctx.Pipe(duplex=True)
        d = float(os.environ.get("NG_ASYNC_CKPT_TEST_DELAY", "0")) if delay is None else delay
        self.proc = ctx.Process(target=_writer_loop, args=(child, d), daemon=True)
        self.proc.start()
        child.close()
        shm = "/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir()
        self.files = [os.path.join(shm, f"ng-ckpt-{os.getpid()}-{id(self):x}-{k}") for k in range(nbuf)]
        self.sizes = [0] * nbuf
        self.views = [None] * nbuf   # uint8 tensors over the shared files (this process's mapping)
        self.busy = [None] * nbuf    # destination being written from slot k, or None
        self.errors = []

    def _collect(self, block):
        """Takes the writer's answers; block=True waits until at least one slot is free again."""
        while any(b is not None for b in self.busy):
            if not self.conn.poll(1.0 if block else 0):
                if not block:
                    return
                if not self.proc.is_alive():
                    raise RuntimeError("checkpoint writer process died")
                continue
            slot, dest, err = self.conn.recv()
            self.busy[slot] = None
            if err:
                self.errors.append((dest, err))
            if block:
                return

    def _slot_view(self, k, size):
        if self.sizes[k] < size:
            with open(self.files[k], "a+b") as f:
                f.truncate(size)
            self.views[k] = torch.from_file(self.files[k], shared=True, size=size, dtype=torch.uint8)
            self.sizes[k] = size
        return self.views[k]

    def save(self, ck, path):
        self._collect(block=False)
        while None not in self.busy:
            self._collect(block=True)
        k = self.busy.index(None)
        # EMA twins (ema_denoiser.X with denoiser.X's values) are stored once
        sd = ck.get("state_dict", {})
        same_as = {}
        for key, t in sd.items():
            if key.startswith("ema_denoiser.") and torch.is_tensor(t):
                r = sd.get("denoiser." + key[len("ema_denoiser."):])
                if r is t or (torch.is_tensor(r) and r.dtype == t.dtype and r.shape == t.shape and torch.equal(r, t)):
                    same_as[id(t)] = r
        offset, order, size = {}, [], 0
        for t in _leaves(ck):
            src = same_as.get(id(t), t)
            if id(src) not in offset:
                offset[id(src)] = size
                order.append(src)
                size += -(-src.numel() * src.element_size() // 64) * 64  # 64-byte aligned
        view = self._slot_view(k, max(size, 64))
        for t in order:
            n = t.numel() * t.element_size()
            if n:
                o = offset[id(t)]
                view[o:o + n].view(t.dtype).view(t.shape).copy_(t.detach())
        skel = _tree_map(ck, lambda v: _Blob(offset[id(same_as.get(id(v), v))], v.dtype, v.shape)
                         if torch.is_tensor(v) else v)
        self.busy[k] = path
        self.conn.send((k, self.files[k], max(size, 64), skel, path, time.time()))

    def wait(self):
        while any(b is not None for b in self.busy):
            self._collect(block=True)
        if self.errors:
            errs, self.errors = self.errors, []
            raise RuntimeError(f"checkpoint writes failed: {errs}")

    def close(self):
        try:
            self.wait()
        finally:
            try:
                self.conn.send(None)
            except OSError:
                pass
            self.proc.join(timeout=30)
            self.conn.close()
            self.views = [None] * len(self.views)
            for name in self.files:
                if os.path.exists(name):
                    os.unlink(name)


def _leaves(obj):
    out = []
    _tree_map(obj, lambda v: out.append(v) if torch.is_tensor(v) else None)
    return out


def clean_tmp(directory):
    """Removes partial checkpoint files (`*.ckpt.part-<pid>`) left by writers that were killed: those whose process
    no longer exists (a live writer's file is kept)."""
    n = 0
    for p in glob.glob(os.path.join(directory, "*.ckpt.part-*")):
        m = re.search(r"\.part-(\d+)$", p)
        if m and not os.path.exists(f"/proc/{m.group(1)}"):
            os.remove(p)
            n += 1
    return n


# ------------------------------------------------------------------------------------------------------- policies
class CheckpointPolicy:
    """When to save: ms-step files (model only) every `ms_every` steps and at max_steps, last.ckpt (full state) every
    `last_every` steps; never at the step the launch resumed from (reference model_checkpoint.py:42-45). Rank 0
    writes; one line per save."""

    def __init__(self, run_dir, ms_every=0, last_every=0, max_steps=None, writer=None, rank=0):
        self.run_dir, self.ms_every, self.last_every = run_dir, ms_every, last_every
        self.max_steps, self.writer, self.rank = max_steps, writer, rank
        self.resumed_step = None
        os.makedirs(run_dir, exist_ok=True)

    def on_start(self, step):
        self.resumed_step = step

    def due(self, step):
        if step == self.resumed_step or step == 0:
            return []
        out = []
        if (self.ms_every and step % self.ms_every == 0) or (self.max_steps and step == self.max_steps):
            out.append((MS_NAME.format(step=step), False))
        if self.last_every and step % self.last_every == 0:
            out.append(("last.ckpt", True))
        return out

    def maybe_save(self, trainer, ema=None):
        saved = []
        for name, full in self.due(trainer.global_step):
            saved.append(self.save(trainer, name, full, ema))
        return saved

    def save(self, trainer, name, full, ema=None):
        path = os.path.join(self.run_dir, name)
        ck = build_checkpoint(trainer, full, ema)
        if self.rank == 0:
            if self.writer is not None:
                self.writer.save(ck, path)
            else:
                save_sync(ck, path)
            print(f"[ckpt] step {trainer.global_step} ({trainer.global_step * trainer.accum} micro-batches): {name}",
                  flush=True)
        return path


class SaveOnTerm:
    """SIGTERM only sets a flag; every `every` steps the ranks take the MAX of their flags with one all-reduce, so all
    stop at the same step, save last-term.ckpt through the normal path, wait for the write and stop (reference
    src/callbacks/save_on_term.py:21-56)."""

    def __init__(self, every=20, filename="last-term.ckpt", install=True):
        self.every = int(os.environ.get("GPIC_TERM_CHECK_EVERY", every))
        self.filename = filename
        self.flag, self.t_flag, self.done = False, None, False
        if install:
            signal.signal(signal.SIGTERM, self._handler)

    def _handler(self, signum, frame):
        if not self.flag:
            self.flag, self.t_flag = True, time.time()

    def check(self, step, device="cpu"):
        """True when every rank must save and stop at this step (a collective on multi-rank runs)."""
        if self.done or step % self.every:
            return False
        t = torch.tensor([1.0 if self.flag else 0.0], device=device)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if t.item() == 0.0:
            return False
        self.done = True
        return True

    def save_and_stop(self, trainer, policy, ema=None):
        t0 = time.time()
        path = policy.save(trainer, self.filename, True, ema)
        if policy.writer is not None and policy.rank == 0:
            policy.writer.wait()
        if dist.is_available() and dist.is_initialized():
            dist.barrier()
        if policy.rank == 0:
            waited = f"{t0 - self.t_flag:.1f} s after the TERM" if self.t_flag else "TERM on another rank"
            print(f"[save_on_term] step {trainer.global_step}: saved {path} in {time.time() - t0:.1f} s ({waited}); "
                  "stopping", flush=True)
        return path
