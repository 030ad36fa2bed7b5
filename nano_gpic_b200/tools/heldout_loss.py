#!/usr/bin/env python3
"""Held-out loss of ladder checkpoints: the training objective on fixed data, fixed noise and 16 fixed noise levels.

The metric (its definition is shared with reference tools/heldout_loss.py:1-36, :251-277, so that numbers compare):
  levels  t_k = time_shift(sigmoid(P_mean + P_std * Phi^-1((k + 0.5) / 16))), k = 0..15, float64 then float32
  noise   image j of a split draws randn((16, C, H, W)) from a CPU generator seeded SEED * 1_000_003 + j (SEED = 0):
          independent of the batch, the device and the number of workers
  loss    JiT's objective with t and the noise given: x_t = t x + (1 - t) eps, v = (x - x_t) / max(1 - t, t_eps), the
          network's x prediction turned into v the same way, squared error averaged over C, H, W per image; sums in
          float64. A record holds the mean over levels and images (loss_<split>), the 16 level means (loss_<split>_t)
          and the standard error over images of the per-image mean over levels (loss_<split>_se).

How this tool gets there (its own design):
  * A split is a HeldoutSplit: uint8 images, the caption features of all captions back to back, their lengths. Its
    images are visited in order of caption length, so a batch pads little (the order changes only rounding).
  * Noise is made on the host, one batch ahead: while the device works on batch b, a thread pool fills batch b + 1's
    tensor (one task per image, each with its own generator, so the values do not depend on the pool).
  * Several workers share one task list through claim files: a worker owns task i when it is the one that creates
    `<counter>.claims/<i>` (O_CREAT | O_EXCL, atomic on the file system), so every task is done once.
  * Results go to a JSON-lines file through a ResultStore, which knows the keys already done; `work` skips them
    (idempotent), so a crashed or repeated job only adds what is missing.
  * A no-EMA checkpoint keeps the raw weights in its EMA slot as well; when every EMA tensor has the raw tensor's bytes,
    one pass over the raw weights gives both records (marked one_pass).

Subcommands (the reference tool's names, arguments and record fields):
  prep  --n-val N --n-train N --data F --val-glob G --train-shard S --emb-dir D [--val-emb-dir D2]
  list  --data F --out results.jsonl [--ckpt ... | --runs DIR] [--skipped FILE]   tasks without a record, as JSON lines
  work  --data F --out results.jsonl (--ckpt ... | --tasks F --counter F)        computes and appends records
  bench --d 1792 --nb 18 --nt 4                                                   seconds per forward, random weights
"""
import argparse
import glob
import json
import math
import os
import re
import socket
import sys
import time
import traceback
import zipfile
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field

import numpy as np
import torch

NUM_T, SEED, BATCH = 16, 0, 128
SPLITS = ("val", "train", "train_reenc")
IMAGE, PAD_MULTIPLE, TEXT_MAX, EMB_DIM = 256, 8, 320, 2048
WEIGHTS = (("ema", "ema_denoiser."), ("raw", "denoiser."))   # record name -> state-dict prefix
CKPT_NAME = re.compile(r"ms-step=(\d+)\.ckpt")
RUN_NAME = re.compile(r"exp_ladder_(d\d+)")
MODEL_ARGS = ("input_size", "in_channels", "num_groups", "hidden_size", "num_blocks", "num_text_blocks", "patch_size",
              "txt_embed_dim", "txt_max_length", "bottleneck_dim")
LOSS_DEFAULTS = dict(timeshift=1.0, P_mean=-0.8, P_std=0.8, t_eps=0.05)


# ====================================================================================================== the metric
def time_shift_fn(t, timeshift=1.0):
    return t / (t + (1 - t) * timeshift)


def levels(P_mean=-0.8, P_std=0.8, timeshift=1.0, num_t=NUM_T):
    """The num_t noise levels: logit-normal quantiles at (k + 0.5) / num_t, in float64, then float32, then shifted."""
    q = (torch.arange(num_t, dtype=torch.float64) + 0.5) / num_t
    return time_shift_fn(torch.sigmoid(P_mean + P_std * torch.special.ndtri(q)).float(), timeshift)


def image_noise(seed, j, num_t, shape, out=None):
    """Image j's noise at every level: randn((num_t, *shape)) from its own CPU generator."""
    gen = torch.Generator().manual_seed(seed * 1_000_003 + j)
    return torch.randn((num_t, *shape), generator=gen, out=out)


def level_loss(net, x, y, y_mask, t, noise, t_eps=0.05):
    """Per-image loss [B] at one level t (a 0-d tensor), with the noise given."""
    tb = t.reshape(1, 1, 1, 1).to(x.dtype)
    x_t = tb * x + (1 - tb) * noise
    den = (1 - tb).clamp_min(t_eps)
    with torch.no_grad():
        pred = net(x_t, t.expand(x.shape[0]), y, y_mask=y_mask)
    err = (pred.float() - x_t) / den - (x - x_t) / den
    return err.square().mean(dim=(1, 2, 3))


def to_input(u8):
    """[B, H, W, 3] uint8 -> [B, 3, H, W] in [-1, 1] (ToTensor, then Normalize(0.5, 0.5))."""
    return ((u8.permute(0, 3, 1, 2).to(torch.float32) / 255.0) - 0.5) / 0.5


# ========================================================================================================== data
@dataclass
class HeldoutSplit:
    """One data split: images [N, H, W, 3] uint8, caption features [sum of lengths, D] (captions back to back),
    caption lengths [N]; captions pad to the batch's longest, rounded up to pad_multiple, at most text_max_length."""
    img: torch.Tensor
    emb: torch.Tensor
    lens: list
    pad_multiple: int = PAD_MULTIPLE
    text_max_length: int = TEXT_MAX
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        self.lens = [int(n) for n in self.lens]
        self.starts = np.concatenate([[0], np.cumsum(self.lens)[:-1]]).astype(np.int64).tolist()

    def __len__(self):
        return len(self.lens)

    @property
    def image_shape(self):
        return (self.img.shape[3], self.img.shape[1], self.img.shape[2])

    def batches(self, size):
        """Index lists of at most `size` images, in order of caption length (ties by index)."""
        order = sorted(range(len(self)), key=lambda i: (self.lens[i], i))
        return [order[k:k + size] for k in range(0, len(order), size)]

    def captions(self, idx, device):
        """(features [B, T, D] with zeros after each caption, mask [B, T]) of images idx."""
        want = max(self.lens[i] for i in idx)
        T = min(-(-want // self.pad_multiple) * self.pad_multiple, self.text_max_length)
        feats = torch.zeros((len(idx), T, self.emb.shape[1]), dtype=self.emb.dtype)
        mask = torch.zeros((len(idx), T), dtype=torch.bool)
        for row, i in enumerate(idx):
            n = min(self.lens[i], T)
            feats[row, :n] = self.emb[self.starts[i]:self.starts[i] + n]
            mask[row, :n] = True
        return feats.to(device), mask.to(device)

    def images(self, idx, device):
        return to_input(self.img[torch.as_tensor(idx)].to(device))

    @classmethod
    def from_saved(cls, d):
        known = {"img", "emb", "lens", "pad_multiple", "text_max_length", "offs"}
        lens = d["lens"].tolist() if torch.is_tensor(d["lens"]) else list(d["lens"])
        return cls(d["img"], d["emb"], lens, int(d.get("pad_multiple", PAD_MULTIPLE)),
                   int(d.get("text_max_length", TEXT_MAX)), {k: v for k, v in d.items() if k not in known})

    def to_saved(self):
        lens = torch.tensor(self.lens, dtype=torch.int64)
        return dict(self.extra, img=self.img, emb=self.emb, lens=lens, offs=torch.tensor(self.starts),
                    pad_multiple=self.pad_multiple, text_max_length=self.text_max_length)


class NoiseAhead:
    """Iterates the noise tensors [B, num_t, *shape] of the given batches in order, each one made by a thread pool
    while the caller still works on the previous one (one batch of lookahead; each image has its own generator)."""

    def __init__(self, batches, seed, num_t, shape, threads=4, pin=False):
        self.batches, self.seed, self.num_t, self.shape, self.pin = batches, seed, num_t, shape, pin
        self.pool = ThreadPoolExecutor(max(1, threads), thread_name_prefix="heldout-noise")

    def _start(self, idx):
        out = torch.empty((len(idx), self.num_t, *self.shape), pin_memory=self.pin)
        jobs = [self.pool.submit(image_noise, self.seed, j, self.num_t, self.shape, out[r]) for r, j in enumerate(idx)]
        return out, jobs

    def __iter__(self):
        try:
            nxt = self._start(self.batches[0]) if self.batches else None
            for b in range(len(self.batches)):
                out, jobs = nxt
                for job in jobs:
                    job.result()  # re-raises a failed draw here
                nxt = self._start(self.batches[b + 1]) if b + 1 < len(self.batches) else None
                yield out
        finally:
            self.pool.shutdown(wait=True, cancel_futures=True)


@torch.no_grad()
def evaluate(nets, split, ts, seed=SEED, batch=BATCH, device="cpu", threads=4, t_eps=0.05, log=None):
    """{name: {"level_mean": [num_t], "image_mean": [N]}} in float64 for every net in `nets` ({name: module}); all
    nets see the same x_t."""
    N, num_t = len(split), len(ts)
    level_sum = {k: torch.zeros(num_t, dtype=torch.float64) for k in nets}
    per_image = {k: torch.zeros(num_t, N, dtype=torch.float64) for k in nets}
    ts = ts.to(device)
    groups = split.batches(batch)
    pin = torch.device(device).type == "cuda"
    t0 = time.time()
    for b, (idx, noise) in enumerate(zip(groups, NoiseAhead(groups, seed, num_t, split.image_shape, threads, pin))):
        noise = noise.to(device, non_blocking=pin)
        x = split.images(idx, device)
        y, mask = split.captions(idx, device)
        cols = torch.as_tensor(idx)
        for name, net in nets.items():
            for k in range(num_t):
                vals = level_loss(net, x, y, mask, ts[k], noise[:, k], t_eps).double().cpu()
                level_sum[name][k] += vals.sum()
                per_image[name][k, cols] = vals
        if log is not None and (b + 1) % max(1, len(groups) // 4) == 0:
            log(f"{b + 1}/{len(groups)} batches, {time.time() - t0:.0f} s")
    return {k: {"level_mean": level_sum[k] / N, "image_mean": per_image[k].mean(0)} for k in nets}


# ======================================================================================================= models
def run_config(run_dir):
    """(denoiser kwargs, loss settings) of a run, from the configurations its launches saved
    (config-TrainerFn.FITTING-<stamp>.yaml); every launch must agree on both."""
    import yaml
    seen = {}
    for path in sorted(glob.glob(os.path.join(run_dir, "config-TrainerFn.FITTING-*.yaml"))):
        with open(path) as f:
            model = yaml.safe_load(f)["model"]
        den = {k: v for k, v in model["denoiser"]["init_args"].items() if k in MODEL_ARGS}
        trainer_args = model.get("diffusion_trainer", {}).get("init_args", {})
        loss = {k: trainer_args.get(k, v) for k, v in LOSS_DEFAULTS.items()}
        seen[json.dumps([den, loss], sort_keys=True)] = (den, loss)
    if not seen:
        raise FileNotFoundError(f"{run_dir}: no config-TrainerFn.FITTING-*.yaml")
    if len(seen) > 1:
        raise ValueError(f"{run_dir}: its launches disagree on the model or the loss: {list(seen)}")
    return next(iter(seen.values()))


def build_denoiser(kw, state_dict, prefix, device):
    """This package's JiT_T2I(**kw) on `device`, fp32, eval mode, with every tensor under `prefix` loaded strictly."""
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    n = len(prefix)
    weights = {k[n:]: v for k, v in state_dict.items() if k.startswith(prefix)}
    with torch.no_grad():
        net = JiT_T2I(**{k: v for k, v in kw.items() if k in MODEL_ARGS}).to(device)
    missing, unexpected = net.load_state_dict(weights, strict=False)
    if missing or unexpected:
        raise KeyError(f"{prefix}*: missing {missing[:5]}, unexpected {unexpected[:5]}")
    return net.float().eval()


def ema_is_raw(state_dict):
    """True when the EMA slot is a byte-for-byte copy of the raw weights (same keys, dtypes, shapes and bytes)."""
    ema = {k[len("ema_denoiser."):]: v for k, v in state_dict.items() if k.startswith("ema_denoiser.")}
    raw = {k[len("denoiser."):]: v for k, v in state_dict.items() if k.startswith("denoiser.")}
    if not ema or set(ema) != set(raw):
        return False

    def as_bytes(t):
        return t.detach().contiguous().reshape(-1).view(torch.uint8)

    for k, e in ema.items():
        r = raw[k]
        if e.dtype != r.dtype or e.shape != r.shape:
            return False
        if e.numel() and not torch.equal(as_bytes(e), as_bytes(r)):
            return False
    return True


# ==================================================================================================== bookkeeping
def task_of(ckpt):
    """The task spec of one ms checkpoint: its absolute path, run root, ladder size (from exp_ladder_dNNN) and step."""
    path = os.path.abspath(ckpt)
    m = CKPT_NAME.fullmatch(os.path.basename(path))
    if m is None:
        raise ValueError(f"not an ms checkpoint (<run>/ms-step=<step>.ckpt): {ckpt}")
    run = os.path.dirname(path)
    r = RUN_NAME.fullmatch(os.path.basename(run))
    return dict(ckpt=path, run_root=os.path.dirname(run), size=r.group(1) if r else None, step=int(m.group(1)))


def find_checkpoints(runs):
    """Every <runs>/exp_ladder_d*/ms-step=*.ckpt, sorted by run and step."""
    found = []
    for run in sorted(e.path for e in os.scandir(runs) if e.is_dir() and RUN_NAME.fullmatch(e.name)):
        found += [e.path for e in os.scandir(run) if e.is_file() and CKPT_NAME.fullmatch(e.name)]
    return sorted(found, key=lambda p: (os.path.dirname(p), int(CKPT_NAME.fullmatch(os.path.basename(p)).group(1))))


def whole_file(path):
    """A checkpoint file is whole once its zip directory (written last by torch.save) is readable."""
    try:
        return zipfile.is_zipfile(path)
    except OSError:
        return False


class ResultStore:
    """The JSON-lines output: the set of (checkpoint, weights, n_val, n_train, num_t, seed, data) already recorded,
    and appends of whole lines (one write per batch of records under an exclusive flock, then fsync)."""

    KEY = ("ckpt", "weights", "n_val", "n_train", "num_t", "seed", "data")

    def __init__(self, path):
        self.path = path

    def done(self):
        keys = set()
        if not os.path.exists(self.path):
            return keys
        with open(self.path) as f:
            for line in f:
                try:
                    rec = json.loads(line)
                    keys.add(tuple(rec[k] for k in self.KEY))
                except (json.JSONDecodeError, KeyError):
                    continue  # a torn or foreign line counts as not done
        return keys

    def missing(self, task, n_val, n_train, data_tag):
        have = self.done()
        return [w for w, _ in WEIGHTS if (task["ckpt"], w, n_val, n_train, NUM_T, SEED, data_tag) not in have]

    def add(self, records):
        import fcntl
        blob = "".join(json.dumps(r) + "\n" for r in records).encode()
        fd = os.open(self.path, os.O_WRONLY | os.O_APPEND | os.O_CREAT, 0o644)
        try:
            fcntl.flock(fd, fcntl.LOCK_EX)
            os.write(fd, blob)
            os.fsync(fd)
        finally:
            os.close(fd)


class ClaimDir:
    """Task hand-out between workers that share a task list: task i belongs to the worker that creates the file
    `<dir>/<i>` (O_CREAT | O_EXCL). Each worker scans upwards from its last claim, so every task goes to one worker."""

    def __init__(self, path):
        self.dir = path
        os.makedirs(path, exist_ok=True)
        self.pos = 0

    def next(self, n_tasks):
        while self.pos < n_tasks:
            i, self.pos = self.pos, self.pos + 1
            try:
                os.close(os.open(os.path.join(self.dir, str(i)), os.O_CREAT | os.O_EXCL | os.O_WRONLY, 0o644))
                return i
            except FileExistsError:
                continue
        return None


def evaluate_task(task, weights, data, opts, device):
    """The records of one checkpoint for the asked weights (a subset of ema, raw)."""
    t0 = time.time()
    kw, loss = run_config(os.path.dirname(task["ckpt"]))
    ck = torch.load(task["ckpt"], map_location="cpu", mmap=True, weights_only=False)
    if ck.get("global_step") != task["step"]:
        raise ValueError(f"{task['ckpt']}: global_step {ck.get('global_step')} != {task['step']}")
    sd = ck["state_dict"]
    one_pass = set(weights) == {"ema", "raw"} and ema_is_raw(sd)
    prefix = dict(WEIGHTS)
    nets = {w: build_denoiser(kw, sd, prefix[w], device) for w in (["raw"] if one_pass else weights)}
    del ck, sd
    ts = levels(loss["P_mean"], loss["P_std"], loss["timeshift"])
    scores = {s: evaluate(nets, data[s], ts, SEED, opts.batch, device, opts.threads, loss["t_eps"])
              for s in opts.splits}
    cuda = torch.device(device).type == "cuda"
    common = dict(n_val=opts.n_val, n_train=opts.n_train, num_t=NUM_T, seed=SEED, data=data["tag"], t=ts.tolist(),
                  d=kw.get("hidden_size"), nb=kw.get("num_blocks"), nt=kw.get("num_text_blocks"))
    out = []
    for w in weights:
        rec = dict(task, weights=w, **common)
        for s in opts.splits:
            res = scores[s]["raw" if one_pass else w]
            lm, im = res["level_mean"], res["image_mean"]
            rec[f"loss_{s}"] = float(lm.mean())
            rec[f"loss_{s}_t"] = lm.tolist()
            rec[f"loss_{s}_se"] = float(im.std() / math.sqrt(im.numel()))
        rec.update(elapsed_s=round(time.time() - t0, 1), one_pass=one_pass, weights_in_task=list(weights),
                   gpu=torch.cuda.get_device_name(device) if cuda else "cpu", host=socket.gethostname(),
                   time=time.strftime("%Y-%m-%dT%H:%M:%S"), framework="nano_gpic_b200")
        out.append(rec)
    return out


# ====================================================================================================== commands
def load_data(path):
    raw = torch.load(path, map_location="cpu", weights_only=False)
    data = {name: HeldoutSplit.from_saved(raw[name]) for name in SPLITS if name in raw}
    data.update(tag=os.path.splitext(os.path.basename(path))[0], n_val=raw.get("n_val"), n_train=raw.get("n_train"))
    return data


def cmd_prep(a):
    from nano_gpic_b200.data.augment import decode_center_u8
    from nano_gpic_b200.data.tars import gpic_samples
    from nano_gpic_b200.data.text_cache import TextCache

    def first(paths, n):
        got = []
        for p in paths:
            for s in gpic_samples(p):
                got.append(s)
                if len(got) == n:
                    return got
        raise RuntimeError(f"only {len(got)} samples in {len(paths)} shards, {n} asked")

    def split_of(samples, cache):
        embs = [cache.read(s["shard"][:-len(".tar")], s["key"]) for s in samples]
        img = torch.from_numpy(np.stack([decode_center_u8(s["image"], IMAGE) for s in samples]))
        return HeldoutSplit(img, torch.cat(embs).contiguous(), [len(e) for e in embs],
                            extra=dict(keys=[s["key"] for s in samples], captions=[s["caption"] for s in samples]))

    val = split_of(first(sorted(glob.glob(a.val_glob)), a.n_val), TextCache(a.val_emb_dir or a.emb_dir))
    train = split_of(first([a.train_shard], a.n_train), TextCache(a.emb_dir))
    blob = dict(version=1, n_val=a.n_val, n_train=a.n_train, val=val.to_saved(), train=train.to_saved(),
                train_shard=os.path.basename(a.train_shard), created=time.strftime("%Y-%m-%dT%H:%M:%S"))
    os.makedirs(os.path.dirname(os.path.abspath(a.data)), exist_ok=True)
    part = f"{a.data}.part-{os.getpid()}"
    torch.save(blob, part)
    os.replace(part, a.data)
    print(f"[prep] {a.data}: {a.n_val} val + {a.n_train} train images", flush=True)


def cmd_list(a):
    tag = os.path.splitext(os.path.basename(a.data))[0]
    store = ResultStore(a.out)
    paths = a.ckpt if a.ckpt else find_checkpoints(a.runs)
    listed, young = 0, []
    for p in paths:
        if time.time() - os.path.getmtime(p) < a.min_age and not whole_file(p):
            young.append(os.path.abspath(p))  # still being written: the next listing will have it
            continue
        task = task_of(p)
        if store.missing(task, a.n_val, a.n_train, tag):
            print(json.dumps(task))
            listed += 1
    if a.skipped:
        with open(a.skipped, "w") as f:
            f.writelines(p + "\n" for p in young)
    print(f"[list] {listed} tasks; {len(young)} checkpoints still being written left out", file=sys.stderr, flush=True)


def cmd_work(a):
    device = "cpu" if a.device == "cpu" else f"cuda:{a.gpu}"
    if device != "cpu":
        torch.cuda.set_device(a.gpu)
    data = load_data(a.data)
    store = ResultStore(a.out)
    if a.tasks:
        with open(a.tasks) as f:
            tasks = [json.loads(line) for line in f if line.strip()]
        claims = ClaimDir(a.counter + ".claims")
        pick = lambda: claims.next(len(tasks))
    else:
        tasks = [task_of(c) for c in a.ckpt]
        order = iter(range(len(tasks)))
        pick = lambda: next(order, None)
    done = failed = 0
    while (i := pick()) is not None:
        task = tasks[i]
        weights = store.missing(task, a.n_val, a.n_train, data["tag"])
        if not weights:
            continue
        try:
            store.add(evaluate_task(task, weights, data, a, device))
            done += 1
        except Exception:
            failed += 1
            print(f"[heldout] {task['ckpt']} failed:\n{traceback.format_exc()}", flush=True)
    print(f"[heldout] {done} checkpoints done, {failed} failed", flush=True)
    return 1 if failed else 0


def cmd_bench(a):
    from nano_gpic_b200.config.ladder import fwd_flops
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    torch.cuda.set_device(a.gpu)
    net = JiT_T2I(input_size=IMAGE, in_channels=3, num_groups=a.d // 64, hidden_size=a.d, num_blocks=a.nb,
                  num_text_blocks=a.nt, patch_size=16, txt_embed_dim=EMB_DIM, txt_max_length=TEXT_MAX,
                  bottleneck_dim=256).cuda().eval()
    x = torch.rand(a.batch, 3, IMAGE, IMAGE, device="cuda") * 2 - 1
    y = torch.randn(a.batch, a.T, EMB_DIM, device="cuda").bfloat16()
    mask = torch.ones(a.batch, a.T, dtype=torch.bool, device="cuda")
    noise, t = torch.randn_like(x), torch.tensor(0.5, device="cuda")
    run = lambda: level_loss(net, x, y, mask, t, noise)
    for _ in range(3):
        run()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(a.iters):
        run()
    end.record()
    torch.cuda.synchronize()
    sec = start.elapsed_time(end) / 1e3 / a.iters
    images = a.n_val + a.n_train
    print(json.dumps(dict(d=a.d, nb=a.nb, nt=a.nt, batch=a.batch, T=a.T, s_per_forward=round(sec, 4),
                          tflops=round(a.batch * fwd_flops(a.d, a.nb, a.nt, a.T) / sec / 1e12, 1),
                          gpu=torch.cuda.get_device_name(), images=images,
                          compute_min_per_ckpt=round(2 * images * NUM_T / a.batch * sec / 60, 2))), flush=True)


def parser():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    cmds = {name: sub.add_parser(name) for name in ("prep", "list", "work", "bench")}
    for p in cmds.values():
        p.add_argument("--n-val", type=int, default=3072)
        p.add_argument("--n-train", type=int, default=3072)
    for name in ("prep", "list", "work"):
        cmds[name].add_argument("--data", required=True)
    p = cmds["prep"]
    p.add_argument("--val-glob", required=True)
    p.add_argument("--train-shard", required=True)
    p.add_argument("--emb-dir", required=True)
    p.add_argument("--val-emb-dir", default=None)
    for name in ("list", "work"):
        cmds[name].add_argument("--out", required=True)
        cmds[name].add_argument("--ckpt", nargs="*", default=None)
    p = cmds["list"]
    p.add_argument("--runs", default=".")
    p.add_argument("--min-age", type=float, default=600)
    p.add_argument("--skipped", default=None)
    p = cmds["work"]
    p.add_argument("--tasks", default=None)
    p.add_argument("--counter", default=None)
    p.add_argument("--gpu", type=int, default=0)
    p.add_argument("--device", default="cuda", choices=("cuda", "cpu"))
    p.add_argument("--batch", type=int, default=BATCH)
    p.add_argument("--threads", type=int, default=6)
    p.add_argument("--splits", default="val,train", type=lambda s: s.split(","))
    p = cmds["bench"]
    for k, v in (("d", 1792), ("nb", 18), ("nt", 4), ("T", 56), ("iters", 10), ("gpu", 0), ("batch", BATCH)):
        p.add_argument(f"--{k}", type=int, default=v)
    return ap


def main(argv=None):
    a = parser().parse_args(argv)
    if a.cmd == "work" and not ((a.tasks and a.counter and not a.ckpt) or (a.ckpt and not a.tasks)):
        raise SystemExit("work: give --ckpt ..., or --tasks FILE with --counter FILE")
    return {"prep": cmd_prep, "list": cmd_list, "work": cmd_work, "bench": cmd_bench}[a.cmd](a)


if __name__ == "__main__":
    sys.exit(main() or 0)
