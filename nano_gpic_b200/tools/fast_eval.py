"""Sample quality against reference statistics, feature extraction sharded over GPUs (reference tools/fast_eval.py,
gpic_eval/eval.py:287-404).

    torchrun --nproc-per-node N -m nano_gpic_b200.tools.fast_eval SAMPLES.npz REF.npz OUT.json [--batch 256]

SAMPLES: uint8 NHWC images (.npy, or .npz with arr_0, as SaveImagesHook writes). REF: reference statistics with
<backend>_mu / <backend>_sigma (Frechet distance) and/or <backend>_embeddings (PRDC, MMD). Each rank extracts features
of a contiguous slice, rank 0 gathers them in image order (all_gather_object) and computes the metrics
(nano_gpic_b200.eval.metrics). Backends (--backend):
  dino       bicubic resize to 224, ImageNet normalisation, DINOv2 ViT-L/14 from the local torch hub cache (no download
             is attempted); keys dino_*
  inception  the TF-Inception pool_3 features (nano_gpic_b200.eval.inception, weights from --inception-weights or
             GPIC_INCEPTION_WEIGHTS), batches of 125 as the reference's tools/official_inception_sharded.py; keys
             inception_*; the result keys carry the inception_ prefix as the reference's output does
--features FILE.npy skips the extractor.
"""
import argparse
import json
import os
import time

import numpy as np
import torch
import torch.distributed as dist

MEAN = torch.tensor([0.485, 0.456, 0.406]).view(1, 3, 1, 1)
STD = torch.tensor([0.229, 0.224, 0.225]).view(1, 3, 1, 1)


def preprocess(u8, size=224):
    x = torch.from_numpy(np.ascontiguousarray(u8)).permute(0, 3, 1, 2).float() / 255.0
    x = torch.nn.functional.interpolate(x, size=(size, size), mode="bicubic", align_corners=False, antialias=True)
    return (x.clamp(0, 1) - MEAN) / STD


def dinov2(device, repo="facebookresearch/dinov2", name="dinov2_vitl14"):
    hub = torch.hub.get_dir()
    local = os.path.join(hub, repo.replace("/", "_") + "_main")
    if not os.path.isdir(local):
        raise FileNotFoundError(f"DINOv2 is not in the torch hub cache ({local}); pass --features or populate the "
                                "cache on a machine with network access")
    return torch.hub.load(local, name, source="local").to(device).eval()


@torch.no_grad()
def extract(arr, lo, hi, model, device, batch=256):
    out = []
    for s in range(lo, hi, batch):
        x = preprocess(np.asarray(arr[s:min(s + batch, hi)])).to(device)
        out.append(model(x).float().cpu().numpy())
    return np.concatenate(out) if out else np.zeros((0, 1), np.float32)


@torch.no_grad()
def extract_inception(arr, lo, hi, model, device, batch=125):
    out = [model(torch.from_numpy(np.ascontiguousarray(arr[s:min(s + batch, hi)])).to(device)).float().cpu().numpy()
           for s in range(lo, hi, batch)]
    return np.concatenate(out) if out else np.zeros((0, 2048), np.float32)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("samples")
    ap.add_argument("ref")
    ap.add_argument("out")
    ap.add_argument("--batch", type=int, default=None, help="images per extractor batch (dino 256, inception 125)")
    ap.add_argument("--backend", default="dino", choices=["dino", "inception"])
    ap.add_argument("--inception-weights", default=None)
    ap.add_argument("--features", default=None, help="precomputed sample features (.npy) instead of the extractor")
    a = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo")
    rank = dist.get_rank() if dist.is_initialized() else 0
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))) if torch.cuda.is_available() else \
        torch.device("cpu")
    t0 = time.time()
    if a.features:
        feats = np.load(a.features) if rank == 0 else None
    else:
        arr = np.load(a.samples, mmap_mode="r") if a.samples.endswith(".npy") else np.load(a.samples)["arr_0"]
        n = arr.shape[0]
        if a.backend == "inception":  # whole batches of 125 per rank, so every feature is the one-pass feature
            bs = a.batch or 125
            nb = (n + bs - 1) // bs
            lo, hi = min(n, rank * nb // world * bs), min(n, (rank + 1) * nb // world * bs)
            from ..eval.inception import FIDInception
            f = extract_inception(arr, lo, hi, FIDInception.from_file(a.inception_weights).to(dev), dev, bs)
        else:
            lo, hi = rank * n // world, (rank + 1) * n // world
            f = extract(arr, lo, hi, dinov2(dev), dev, a.batch or 256)
        parts = [None] * world
        if world > 1:
            dist.all_gather_object(parts, (lo, f))
        else:
            parts = [(lo, f)]
        feats = np.concatenate([p for _, p in sorted(parts, key=lambda t: t[0])]) if rank == 0 else None
    if rank == 0:
        from ..eval.metrics import evaluate
        ref = np.load(a.ref)
        k = a.backend
        res = evaluate(feats, real=ref[f"{k}_embeddings"] if f"{k}_embeddings" in ref.files else None,
                       ref_mu=ref[f"{k}_mu"] if f"{k}_mu" in ref.files else None,
                       ref_sigma=ref[f"{k}_sigma"] if f"{k}_sigma" in ref.files else None)
        if k == "inception":
            res = {f"inception_{name}": v for name, v in res.items()}
        res.update(world=world, total_s=time.time() - t0)
        with open(a.out, "w") as fh:
            json.dump(res, fh, indent=1)
        print(json.dumps(res, indent=1))
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
