"""Reading webdataset-style tar shards without webdataset: members grouped into samples by key.

A member `dir/abc.def.jpg` belongs to sample `dir/abc` with suffix `def.jpg` lower-cased (the key runs to the first dot
of the file name), and consecutive members of one key form a sample, as webdataset's tar iterator groups them
(reference tools/heldout_loss.py:90-107 uses it the same way).
"""
import json
import os
import tarfile

IMAGE_SUFFIXES = ("jpg", "jpeg", "png", "webp")


def split_key(name):
    d, f = os.path.split(name)
    if "." not in f:
        return None, None
    i = f.index(".")
    return os.path.join(d, f[:i]) if d else f[:i], f[i + 1:].lower()


def tar_groups(path):
    """(key, {suffix: bytes}) in tar order."""
    key, cur = None, {}
    with tarfile.open(path) as tar:
        for m in tar:
            if not m.isfile():
                continue
            k, ext = split_key(m.name)
            if k is None:
                continue
            if k != key or ext in cur:
                if key is not None:
                    yield key, cur
                key, cur = k, {}
            cur[ext] = tar.extractfile(m).read()
    if key is not None:
        yield key, cur


def gpic_samples(path):
    """GPIC samples of a shard: dicts with key, image bytes, caption, caption_type (the training filters: a sample
    needs an image, a caption and a caption type)."""
    for key, d in tar_groups(path):
        img = next((e for e in IMAGE_SUFFIXES if e in d), None)
        meta = json.loads(d["json"]) if "json" in d else {}
        if img is None or "caption" not in meta or "caption_type" not in meta:
            continue
        yield dict(key=key, shard=os.path.basename(path), image=d[img], caption=meta["caption"],
                   caption_type=meta["caption_type"])
