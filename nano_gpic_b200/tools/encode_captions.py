"""Builds the text-encoder cache for GPIC shards (reference tools/encode_captions.py:1-113): every caption of each tar
is tokenized and encoded once with the training path's encoder (Qwen3TextEncoder: right padding to the longest caption
of a length-sorted batch, rounded up to 8, at most 320 tokens, bf16); the real tokens' outputs go to <shard>.emb and
the keys/offsets/lengths to <shard>.idx.npz (atomic renames); null.pt holds the null caption (one EOS token).
Shards are split over ranks (torchrun); existing complete shards are skipped.

    torchrun --nproc-per-node 8 -m nano_gpic_b200.tools.encode_captions --tar-dir DATA/train \
        --pattern "gpic_train_{00000..07999}.tar" --out DATA/train_emb_qwen3_1.7b --weights Qwen3-1.7B-dir
"""
import argparse
import os

import torch

from ..data.gpic import expand_pattern
from ..data.tars import gpic_samples
from ..data.text_cache import write_shard


def encode_shard(encoder, tar_path, out_dir, batch=64, max_length=320):
    name = os.path.basename(tar_path)[:-len(".tar")]
    keys, caps = [], []
    for s in gpic_samples(tar_path):
        keys.append(s["key"])
        caps.append(s["caption"])
    order = sorted(range(len(caps)), key=lambda i: len(caps[i]))
    embs = [None] * len(caps)
    for b in range(0, len(order), batch):
        idx = order[b:b + batch]
        ids, mask = encoder.tokenize([caps[i] for i in idx])
        out, mask = encoder.encode(ids[:, :max_length], mask[:, :max_length])
        for j, i in enumerate(idx):
            embs[i] = out[j, :int(mask[j].sum())].cpu()
    write_shard(out_dir, name, keys, embs)
    return len(keys)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tar-dir", required=True)
    ap.add_argument("--pattern", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--weights", required=True, help="local Hugging Face Qwen3 directory")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--max-length", type=int, default=320)
    a = ap.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))) if torch.cuda.is_available() else "cpu"
    from ..models.conditioner import Qwen3TextEncoder
    enc = Qwen3TextEncoder(a.weights, embed_dim=2048, max_length=a.max_length, device=dev)
    os.makedirs(a.out, exist_ok=True)
    if rank == 0 and not os.path.exists(os.path.join(a.out, "null.pt")):
        torch.save(enc.null().cpu(), os.path.join(a.out, "null.pt"))
    tars = expand_pattern(os.path.join(a.tar_dir, a.pattern))[rank::world]
    for t in tars:
        name = os.path.basename(t)[:-len(".tar")]
        if os.path.exists(os.path.join(a.out, name + ".idx.npz")):
            continue
        n = encode_shard(enc, t, a.out, a.batch, a.max_length)
        print(f"[rank {rank}] {name}: {n} captions", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
