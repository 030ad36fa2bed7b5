"""Sample quality against reference statistics, feature extraction sharded over GPUs (reference tools/fast_eval.py,
gpic_eval/eval.py:287-404).

    torchrun --nproc-per-node N -m nano_gpic_b200.tools.fast_eval SAMPLES.npz REF.npz OUT.json [--batch 256]

SAMPLES: uint8 NHWC images (.npy, or .npz with arr_0, as SaveImagesHook writes). REF: reference statistics with
dino_mu / dino_sigma (Frechet distance) and/or dino_embeddings (PRDC, MMD). Each rank extracts features of a
contiguous slice (bicubic resize to 224, ImageNet normalisation, a DINOv2 ViT-L/14 from the local torch hub cache; no
download is attempted), rank 0 gathers them in image order (all_gather_object) and computes the metrics
(nano_gpic_b200.eval.metrics). --features FILE.npy skips the extractor.
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


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("samples")
    ap.add_argument("ref")
    ap.add_argument("out")
    ap.add_argument("--batch", type=int, default=256)
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
        lo, hi = rank * n // world, (rank + 1) * n // world
        f = extract(arr, lo, hi, dinov2(dev), dev, a.batch)
        parts = [None] * world
        if world > 1:
            dist.all_gather_object(parts, (lo, f))
        else:
            parts = [(lo, f)]
        feats = np.concatenate([p for _, p in sorted(parts, key=lambda t: t[0])]) if rank == 0 else None
    if rank == 0:
        from ..eval.metrics import evaluate
        ref = np.load(a.ref)
        res = evaluate(feats, real=ref["dino_embeddings"] if "dino_embeddings" in ref.files else None,
                       ref_mu=ref["dino_mu"] if "dino_mu" in ref.files else None,
                       ref_sigma=ref["dino_sigma"] if "dino_sigma" in ref.files else None)
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
