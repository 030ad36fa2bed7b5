"""Verifies a text-encoder cache against its tar shards (reference tools/check_text_cache.py:1-60): every tar key has
an index entry, offsets are contiguous, the .emb size equals the tokens x dim x 2 bytes, lengths lie in [1, 320], and
null.pt is [1, 1, dim] bf16. Exit 1 with a report when anything is off.

    python -m nano_gpic_b200.tools.check_text_cache --tar-dir DATA/train --pattern "gpic_train_{00000..00010}.tar" \
        --emb-dir DATA/train_emb_qwen3_1.7b
"""
import argparse
import os
import sys

import numpy as np
import torch

from ..data.gpic import expand_pattern
from ..data.tars import gpic_samples
from ..data.text_cache import EMB_DIM


def check_shard(tar_path, emb_dir, dim=EMB_DIM, max_len=320):
    name = os.path.basename(tar_path)[:-len(".tar")]
    idx_path, emb_path = os.path.join(emb_dir, name + ".idx.npz"), os.path.join(emb_dir, name + ".emb")
    if not (os.path.exists(idx_path) and os.path.exists(emb_path)):
        return [f"{name}: missing cache files"]
    problems = []
    with np.load(idx_path) as z:
        keys, offs, lens = z["keys"].tolist(), z["offsets"], z["lengths"]
    if len(set(keys)) != len(keys):
        problems.append(f"{name}: duplicate keys")
    if len(lens) and (offs[0] != 0 or np.any(offs[1:] != np.cumsum(lens)[:-1])):
        problems.append(f"{name}: offsets are not contiguous")
    if len(lens) and (lens.min() < 1 or lens.max() > max_len):
        problems.append(f"{name}: lengths outside [1, {max_len}]")
    size = os.path.getsize(emb_path)
    if size != int(lens.sum()) * dim * 2:
        problems.append(f"{name}: {size} bytes, expected {int(lens.sum()) * dim * 2}")
    tar_keys = {s["key"] for s in gpic_samples(tar_path)}
    missing = tar_keys - set(keys)
    if missing:
        problems.append(f"{name}: {len(missing)} tar samples without cached outputs (e.g. {sorted(missing)[:3]})")
    return problems


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tar-dir", required=True)
    ap.add_argument("--pattern", required=True)
    ap.add_argument("--emb-dir", required=True)
    a = ap.parse_args(argv)
    problems = []
    null = os.path.join(a.emb_dir, "null.pt")
    if not os.path.exists(null):
        problems.append("null.pt missing")
    else:
        t = torch.load(null, map_location="cpu", weights_only=True)
        if t.dtype != torch.bfloat16 or t.shape != (1, 1, EMB_DIM):
            problems.append(f"null.pt is {t.dtype} {tuple(t.shape)}")
    tars = expand_pattern(os.path.join(a.tar_dir, a.pattern))
    for t in tars:
        problems += check_shard(t, a.emb_dir)
    for p in problems:
        print(p)
    print(f"{len(tars)} shards checked: " + ("OK" if not problems else f"{len(problems)} problems"))
    return 1 if problems else 0


if __name__ == "__main__":
    sys.exit(main())
