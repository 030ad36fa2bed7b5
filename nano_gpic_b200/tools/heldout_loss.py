#!/usr/bin/env python3
"""Held-out loss of ladder checkpoints: the training objective on fixed data, fixed noise and 16 fixed noise levels.

The definition (reference tools/heldout_loss.py:1-36, :251-277):
  t_k   = time_shift(sigmoid(P_mean + P_std * Phi^-1((k + 0.5) / 16))), k = 0..15, computed in float64, then float32
  noise = image j of a split draws randn((16, C, H, W)) from a CPU generator seeded SEED * 1_000_003 + j (SEED = 0),
          independent of batch, GPU and GPU count
  loss  = the JiT objective (x_t = t x + (1 - t) eps, v-space squared error, mean over C, H, W per image), per level,
          summed in float64; the record holds the mean over levels and images, the 16 level means and the standard
          error over images
Images are batched in order of caption length (the order changes only rounding). A checkpoint whose EMA slot holds the
raw weights bit for bit is evaluated once for both records (one_pass).

Subcommands (same names and output fields as the reference):
  prep  --n-val N --n-train N --val-glob G --train-shard S --emb-dir D [--val-emb-dir D2]   -> data file
  list  --out results.jsonl [--ckpt ...]        the checkpoints that lack a record
  work  --out results.jsonl --data F (--ckpt ... | --tasks F --counter F)   computes records (appends JSON lines)
  bench --d 1792 --nb 18 --nt 4                 seconds per forward of a random model
"""
import argparse
import fcntl
import glob
import json
import math
import os
import queue
import re
import socket
import sys
import threading
import time
import traceback
import zipfile

import numpy as np
import torch

NUM_T, SEED, BATCH = 16, 0, 128
SPLITS = ("val", "train", "train_reenc")
IMAGE, PAD_MULTIPLE, TEXT_MAX, EMB_DIM = 256, 8, 320, 2048
WEIGHTS = (("ema", "ema_denoiser."), ("raw", "denoiser."))
CKPT_RE = re.compile(r"ms-step=(\d+)\.ckpt")
RUN_RE = re.compile(r"exp_ladder_(d\d+)")


# ------------------------------------------------------------------------------------------------------------ loss
def time_shift_fn(t, timeshift=1.0):
    return t / (t + (1 - t) * timeshift)


def levels(P_mean=-0.8, P_std=0.8, timeshift=1.0, num_t=NUM_T):
    q = (torch.arange(num_t, dtype=torch.float64) + 0.5) / num_t
    base = torch.sigmoid(P_mean + P_std * torch.special.ndtri(q)).float()
    return time_shift_fn(base, timeshift)


def image_noise(seed, j, num_t, shape, out=None):
    g = torch.Generator().manual_seed(seed * 1_000_003 + j)
    return torch.randn((num_t, *shape), generator=g, out=out)


def level_loss(net, x, y, y_mask, t, noise, t_eps=0.05):
    """Per-image loss at one level t (0-d tensor): the JiT objective with t and the noise given."""
    t = t.expand(x.shape[0])
    tt = t.view(-1, 1, 1, 1)
    x_t = tt * x + noise * (1 - tt)
    den = (1 - tt).clamp_min(t_eps)
    v_t = (x - x_t) / den
    with torch.no_grad():
        pred = net(x_t, t, y, y_mask=y_mask)
    out = (pred.float() - x_t) / den
    return ((out - v_t) ** 2).mean(dim=(1, 2, 3))


def to_input(u8):
    """[B, H, W, 3] uint8 -> x in [-1, 1]: ToTensor + Normalize(0.5, 0.5)."""
    return u8.permute(0, 3, 1, 2).float().div(255).sub(0.5).div(0.5)


def text_batch(split, idx, device):
    lens = [int(split["lens"][i]) for i in idx]
    T = min(-(-max(lens) // split["pad_multiple"]) * split["pad_multiple"], split["text_max_length"])
    emb = split["emb"]
    y = torch.zeros((len(idx), T, emb.shape[1]), dtype=emb.dtype, device=device)
    mask = torch.zeros((len(idx), T), dtype=torch.bool, device=device)
    for r, (i, n) in enumerate(zip(idx, lens)):
        o = int(split["offs"][i])
        y[r, :n] = emb[o:o + n]
        mask[r, :n] = True
    return y, mask


def _noise_feed(batches, seed, num_t, shape, threads, pin):
    """Each batch's noise [B, num_t, *shape], generated one batch ahead in a background thread."""
    from concurrent.futures import ThreadPoolExecutor
    q = queue.Queue(maxsize=1)
    stop = threading.Event()
    B = max(len(i) for i in batches)
    bufs = [torch.empty((B, num_t, *shape), pin_memory=pin) for _ in range(min(3, len(batches)))]

    def produce():
        try:
            with ThreadPoolExecutor(threads) as pool:
                for b, idx in enumerate(batches):
                    buf = bufs[b % len(bufs)][:len(idx)]
                    list(pool.map(lambda r: image_noise(seed, idx[r], num_t, shape, out=buf[r]), range(len(idx))))
                    while not stop.is_set():
                        try:
                            q.put(buf, timeout=1)
                            break
                        except queue.Full:
                            pass
                    if stop.is_set():
                        return
            q.put(None)
        except BaseException as e:
            q.put(e)

    th = threading.Thread(target=produce, daemon=True)
    th.start()
    try:
        while True:
            item = q.get()
            if item is None:
                return
            if isinstance(item, BaseException):
                raise item
            yield item
    finally:
        stop.set()


@torch.no_grad()
def evaluate(nets, split, ts, seed=SEED, batch=BATCH, device="cpu", threads=4, t_eps=0.05, log=None):
    """{name: dict(level_mean [num_t], image_mean [N])} in float64, every net on the same x_t."""
    N, num_t = len(split["lens"]), len(ts)
    shape = tuple(split["img"].shape[i] for i in (3, 1, 2))
    order = split.get("order") or sorted(range(N), key=lambda i: (int(split["lens"][i]), i))
    batches = [order[i:i + batch] for i in range(0, N, batch)]
    sums = {k: torch.zeros(num_t, dtype=torch.float64, device=device) for k in nets}
    per = {k: torch.zeros(N, dtype=torch.float64, device=device) for k in nets}
    ts = ts.to(device)
    pin = torch.device(device).type == "cuda"
    t0 = time.time()
    for b, (idx, noise) in enumerate(zip(batches, _noise_feed(batches, seed, num_t, shape, threads, pin))):
        noise = noise.to(device)
        it = torch.tensor(idx, device=device)
        x = to_input(split["img"][it.cpu()].to(device))
        y, mask = text_batch(split, idx, device)
        for k in range(num_t):
            for name, net in nets.items():
                l = level_loss(net, x, y, mask, ts[k], noise[:, k], t_eps).double()
                sums[name][k] += l.sum()
                per[name].index_add_(0, it, l)
        if log and (b + 1) % max(1, len(batches) // 4) == 0:
            log(f"batch {b + 1}/{len(batches)} {time.time() - t0:.0f} s")
    return {k: dict(level_mean=(sums[k] / N).cpu(), image_mean=(per[k] / num_t).cpu()) for k in nets}


# ------------------------------------------------------------------------------------------------------- models
def run_config(run_dir):
    """Denoiser kwargs and loss settings from the run's saved configs (config-TrainerFn.FITTING-*.yaml)."""
    import yaml
    cfgs = sorted(glob.glob(os.path.join(run_dir, "config-TrainerFn.FITTING-*.yaml")))
    assert cfgs, f"no config-TrainerFn.FITTING-*.yaml in {run_dir}"
    dens, losses = set(), set()
    for c in cfgs:
        with open(c) as f:
            m = yaml.safe_load(f)["model"]
        kw = dict(m["denoiser"]["init_args"])
        ta = m["diffusion_trainer"]["init_args"]
        loss = dict(timeshift=ta.get("timeshift", 1.0), P_mean=ta.get("P_mean", -0.8), P_std=ta.get("P_std", 0.8),
                    t_eps=ta.get("t_eps", 0.05))
        dens.add(json.dumps(kw, sort_keys=True))
        losses.add(json.dumps(loss, sort_keys=True))
    assert len(dens) == 1 and len(losses) == 1, f"{run_dir}: launches differ: {dens} {losses}"
    return json.loads(dens.pop()), json.loads(losses.pop())


def build_denoiser(kw, state_dict, prefix, device):
    """nano_gpic_b200's JiT_T2I(**kw) with the weights under prefix, loaded strictly."""
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    sub = {k[len(prefix):]: v for k, v in state_dict.items() if k.startswith(prefix)}
    kw = {k: v for k, v in kw.items() if k in ("input_size", "in_channels", "num_groups", "hidden_size", "num_blocks",
                                               "num_text_blocks", "patch_size", "txt_embed_dim", "txt_max_length",
                                               "bottleneck_dim")}
    with torch.device("meta"):
        net = JiT_T2I(**kw)
    net.load_state_dict(sub, strict=True, assign=True)
    left = [n for n, t in list(net.named_parameters()) + list(net.named_buffers()) if t.is_meta]
    assert not left, f"tensors without weights: {left[:5]}"
    return net.to(device).float().eval()


_BITS = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}


def twin_weights(sd):
    """True when every ema_denoiser.X holds the bytes of denoiser.X (a no-EMA checkpoint)."""
    ema = {k[len("ema_denoiser."):]: v for k, v in sd.items() if k.startswith("ema_denoiser.")}
    raw = {k[len("denoiser."):]: v for k, v in sd.items() if k.startswith("denoiser.")}
    if not ema or ema.keys() != raw.keys():
        return False
    for k, e in ema.items():
        r = raw[k]
        if (e.dtype, e.shape) != (r.dtype, r.shape) or e.element_size() not in _BITS:
            return False
        if e.numel() == 0 or (e.data_ptr() == r.data_ptr() and e.stride() == r.stride()):
            continue
        i = _BITS[e.element_size()]
        if not torch.equal(e.contiguous().view(i), r.contiguous().view(i)):
            return False
    return True


# -------------------------------------------------------------------------------------------------------- tasks
def spec_of(ckpt):
    ckpt = os.path.abspath(ckpt)
    run_dir = os.path.dirname(ckpt)
    m, r = CKPT_RE.fullmatch(os.path.basename(ckpt)), RUN_RE.fullmatch(os.path.basename(run_dir))
    assert m, f"not <...>/ms-step=<step>.ckpt: {ckpt}"
    return dict(ckpt=ckpt, run_root=os.path.dirname(run_dir), size=r.group(1) if r else None, step=int(m.group(1)))


def done_keys(out):
    keys = set()
    if os.path.exists(out):
        with open(out) as f:
            for line in f:
                if line.strip():
                    try:
                        r = json.loads(line)
                    except json.JSONDecodeError:
                        continue
                    keys.add((r["ckpt"], r["weights"], r["n_val"], r["n_train"], r["num_t"], r["seed"], r["data"]))
    return keys


def complete(path):
    try:
        return zipfile.is_zipfile(path)
    except OSError:
        return False


def claim(counter):
    """The next task index from a shared counter file, under lockf."""
    with open(counter, "a+") as f:
        fcntl.lockf(f, fcntl.LOCK_EX)
        f.seek(0)
        s = f.read().strip()
        i = int(s) if s else 0
        f.seek(0)
        f.truncate()
        f.write(str(i + 1))
        f.flush()
        os.fsync(f.fileno())
        return i


def append_lines(path, recs):
    with open(path, "a") as f:
        fcntl.lockf(f, fcntl.LOCK_EX)
        f.write("".join(json.dumps(r) + "\n" for r in recs))
        f.flush()
        os.fsync(f.fileno())


def run_task(spec, weights, data, a, device):
    t0 = time.time()
    kw, loss = run_config(os.path.dirname(spec["ckpt"]))
    ck = torch.load(spec["ckpt"], map_location="cpu", mmap=True, weights_only=False)
    assert ck["global_step"] == spec["step"], (ck["global_step"], spec["step"])
    prefixes = dict(WEIGHTS)
    one_pass = set(weights) == {"ema", "raw"} and twin_weights(ck["state_dict"])
    nets = {w: build_denoiser(kw, ck["state_dict"], prefixes[w], device) for w in (("raw",) if one_pass else weights)}
    del ck
    ts = levels(loss["P_mean"], loss["P_std"], loss["timeshift"])
    res = {s: evaluate(nets, data[s], ts, SEED, a.batch, device, a.threads, loss["t_eps"]) for s in a.splits}
    recs = []
    for w in weights:
        r = dict(spec, weights=w, n_val=a.n_val, n_train=a.n_train, num_t=NUM_T, seed=SEED, data=data["tag"],
                 t=ts.tolist(), d=kw.get("hidden_size"), nb=kw.get("num_blocks"), nt=kw.get("num_text_blocks"))
        for s in a.splits:
            lm, im = (res[s]["raw" if one_pass else w][k] for k in ("level_mean", "image_mean"))
            r[f"loss_{s}"] = float(lm.mean())
            r[f"loss_{s}_t"] = lm.tolist()
            r[f"loss_{s}_se"] = float(im.std() / math.sqrt(len(im)))
        r.update(elapsed_s=round(time.time() - t0, 1), one_pass=one_pass, weights_in_task=list(weights),
                 gpu=torch.cuda.get_device_name(device) if torch.device(device).type == "cuda" else "cpu",
                 host=socket.gethostname(), time=time.strftime("%Y-%m-%dT%H:%M:%S"), framework="nano_gpic_b200")
        recs.append(r)
    return recs


# ------------------------------------------------------------------------------------------------------ commands
def cmd_prep(a):
    from nano_gpic_b200.data.augment import decode_center_u8
    from nano_gpic_b200.data.tars import gpic_samples
    from nano_gpic_b200.data.text_cache import TextCache

    def read(paths, n):
        out = []
        for p in paths:
            for s in gpic_samples(p):
                out.append(s)
                if len(out) == n:
                    return out
        raise RuntimeError(f"only {len(out)} samples in {len(paths)} shards, {n} asked")

    val = read(sorted(glob.glob(a.val_glob)), a.n_val)
    tr = read([a.train_shard], a.n_train)
    cache = TextCache(a.emb_dir)
    vcache = TextCache(a.val_emb_dir or a.emb_dir)

    def pack(ss, c):
        img = torch.from_numpy(np.stack([decode_center_u8(s["image"], IMAGE) for s in ss]))
        embs = [c.read(s["shard"][:-len(".tar")], s["key"]) for s in ss]
        lens = torch.tensor([len(e) for e in embs], dtype=torch.int64)
        offs = torch.cat([torch.zeros(1, dtype=torch.int64), lens.cumsum(0)[:-1]])
        return dict(img=img, emb=torch.cat(embs).contiguous(), lens=lens, offs=offs, pad_multiple=PAD_MULTIPLE,
                    text_max_length=TEXT_MAX, keys=[s["key"] for s in ss], captions=[s["caption"] for s in ss])
    out = dict(version=1, n_val=a.n_val, n_train=a.n_train, val=pack(val, vcache), train=pack(tr, cache),
               created=time.strftime("%Y-%m-%dT%H:%M:%S"))
    os.makedirs(os.path.dirname(os.path.abspath(a.data)) or ".", exist_ok=True)
    tmp = a.data + f".tmp{os.getpid()}"
    torch.save(out, tmp)
    os.replace(tmp, a.data)
    print(f"[prep] wrote {a.data}", flush=True)


def load_data(path):
    d = torch.load(path, map_location="cpu", weights_only=False)
    for name in SPLITS:
        if name in d:
            s = d[name]
            s["order"] = sorted(range(len(s["lens"])), key=lambda i: (int(s["lens"][i]), i))
    d["tag"] = os.path.basename(path)[:-len(".pt")]
    return d


def cmd_list(a):
    tag = os.path.basename(a.data)[:-len(".pt")]
    done = done_keys(a.out)
    ckpts = a.ckpt or sorted(glob.glob(os.path.join(a.runs, "exp_ladder_d*", "ms-step=*.ckpt")))
    n = 0
    for c in ckpts:
        if time.time() - os.path.getmtime(c) < a.min_age and not complete(c):
            continue
        spec = spec_of(c)
        if any((spec["ckpt"], w, a.n_val, a.n_train, NUM_T, SEED, tag) not in done for w, _ in WEIGHTS):
            print(json.dumps(spec))
            n += 1
    print(f"[list] {n} tasks", file=sys.stderr, flush=True)


def cmd_work(a):
    device = f"cuda:{a.gpu}" if a.device == "cuda" else "cpu"
    if a.device == "cuda":
        torch.cuda.set_device(a.gpu)
    data = load_data(a.data)
    if a.tasks:
        with open(a.tasks) as f:
            tasks = [json.loads(line) for line in f if line.strip()]
        nxt = lambda: claim(a.counter)
    else:
        tasks = [spec_of(c) for c in a.ckpt]
        it = iter(range(len(tasks)))
        nxt = lambda: next(it, len(tasks))
    fails = 0
    while True:
        i = nxt()
        if i >= len(tasks):
            break
        spec = tasks[i]
        done = done_keys(a.out)
        weights = [w for w, _ in WEIGHTS if (spec["ckpt"], w, a.n_val, a.n_train, NUM_T, SEED, data["tag"]) not in done]
        if not weights:
            continue
        try:
            append_lines(a.out, run_task(spec, weights, data, a, device))
        except Exception:
            fails += 1
            print(f"[heldout] FAILED {spec['ckpt']}:\n{traceback.format_exc()}", flush=True)
    return 1 if fails else 0


def cmd_bench(a):
    from nano_gpic_b200.config.ladder import fwd_flops
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    torch.cuda.set_device(a.gpu)
    net = JiT_T2I(input_size=IMAGE, in_channels=3, num_groups=a.d // 64, hidden_size=a.d, num_blocks=a.nb,
                  num_text_blocks=a.nt, patch_size=16, txt_embed_dim=EMB_DIM, txt_max_length=TEXT_MAX,
                  bottleneck_dim=256).cuda().eval()
    B = a.batch
    x = torch.randn(B, 3, IMAGE, IMAGE, device="cuda").clamp(-1, 1)
    y = torch.randn(B, a.T, EMB_DIM, device="cuda").bfloat16()
    mask = torch.ones(B, a.T, dtype=torch.bool, device="cuda")
    noise = torch.randn_like(x)
    t = torch.tensor(0.5, device="cuda")
    for _ in range(3):
        level_loss(net, x, y, mask, t, noise)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        level_loss(net, x, y, mask, t, noise)
    e1.record()
    torch.cuda.synchronize()
    s = e0.elapsed_time(e1) / 1000 / a.iters
    n = a.n_val + a.n_train
    print(json.dumps(dict(d=a.d, nb=a.nb, nt=a.nt, batch=B, T=a.T, s_per_forward=round(s, 4),
                          tflops=round(B * fwd_flops(a.d, a.nb, a.nt, a.T) / s / 1e12, 1),
                          gpu=torch.cuda.get_device_name(), images=n,
                          compute_min_per_ckpt=round(2 * n * NUM_T / B * s / 60, 2))), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("prep", "list", "work", "bench"):
        p = sub.add_parser(name)
        p.add_argument("--n-val", type=int, default=3072)
        p.add_argument("--n-train", type=int, default=3072)
        if name in ("prep", "list", "work"):
            p.add_argument("--data", required=True)
        if name == "prep":
            p.add_argument("--val-glob", required=True)
            p.add_argument("--train-shard", required=True)
            p.add_argument("--emb-dir", required=True)
            p.add_argument("--val-emb-dir", default=None)
        if name in ("list", "work"):
            p.add_argument("--out", required=True)
            p.add_argument("--ckpt", nargs="*", default=None)
        if name == "list":
            p.add_argument("--runs", default=".")
            p.add_argument("--min-age", type=float, default=600)
        if name == "work":
            p.add_argument("--tasks", default=None)
            p.add_argument("--counter", default=None)
            p.add_argument("--gpu", type=int, default=0)
            p.add_argument("--device", default="cuda", choices=("cuda", "cpu"))
            p.add_argument("--batch", type=int, default=BATCH)
            p.add_argument("--threads", type=int, default=6)
            p.add_argument("--splits", default="val,train")
        if name == "bench":
            for k, v in (("d", 1792), ("nb", 18), ("nt", 4), ("T", 56), ("iters", 10), ("gpu", 0), ("batch", BATCH)):
                p.add_argument(f"--{k}", type=int, default=v)
    a = ap.parse_args(argv)
    if a.cmd == "prep":
        return cmd_prep(a)
    if a.cmd == "list":
        return cmd_list(a)
    if a.cmd == "work":
        assert bool(a.tasks) == bool(a.counter) and bool(a.tasks) != bool(a.ckpt), "--tasks with --counter, or --ckpt"
        a.splits = a.splits.split(",")
        return cmd_work(a)
    return cmd_bench(a)


if __name__ == "__main__":
    sys.exit(main() or 0)
