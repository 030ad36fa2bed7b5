"""The text-encoder cache: each shard's real-token encoder outputs as raw bf16 bytes (`<shard>.emb`) plus an index
(`<shard>.idx.npz`: keys, token offsets, lengths), written atomically (reference tools/encode_captions.py:1-113,
src/models/conditioner/cached_text.py). Readers use positioned reads, so worker processes share the file.
"""
import os

import numpy as np
import torch

EMB_DIM = 2048


class TextCache:
    def __init__(self, emb_dir, dim=EMB_DIM):
        self.dir, self.dim = emb_dir, dim
        self._index, self._fd = {}, {}

    def _load(self, shard):
        if shard not in self._index:
            with np.load(os.path.join(self.dir, shard + ".idx.npz")) as z:
                self._index[shard] = dict(zip(z["keys"].tolist(), zip(z["offsets"].tolist(), z["lengths"].tolist())))
            self._fd[shard] = os.open(os.path.join(self.dir, shard + ".emb"), os.O_RDONLY)
        return self._index[shard]

    def length(self, shard, key):
        return self._load(shard)[key][1]

    def read(self, shard, key):
        """[n, dim] bf16 outputs of the caption's real tokens; KeyError when the sample is not cached."""
        off, n = self._load(shard)[key]
        nb = n * self.dim * 2
        raw = os.pread(self._fd[shard], nb, off * self.dim * 2)
        if len(raw) != nb:
            raise IOError(f"{shard}.emb: short read for {key} ({len(raw)} of {nb} bytes)")
        return torch.frombuffer(bytearray(raw), dtype=torch.bfloat16).view(n, self.dim)

    def null(self):
        """The null caption (one EOS token) from null.pt, [1, 1, dim] bf16."""
        return torch.load(os.path.join(self.dir, "null.pt"), map_location="cpu", weights_only=True)

    def close(self):
        for fd in self._fd.values():
            os.close(fd)
        self._fd.clear()


def write_shard(emb_dir, shard, keys, embs):
    """Writes one shard's cache: embs is a list of [n_i, dim] bf16 tensors in key order. Atomic (tmp + rename)."""
    os.makedirs(emb_dir, exist_ok=True)
    lens = np.array([int(e.shape[0]) for e in embs], dtype=np.int64)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    emb_path, idx_path = os.path.join(emb_dir, shard + ".emb"), os.path.join(emb_dir, shard + ".idx.npz")
    tmp = emb_path + f".tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        for e in embs:
            f.write(e.contiguous().to(torch.bfloat16).view(torch.int16).numpy().tobytes())
    itmp = idx_path + f".tmp{os.getpid()}.npz"
    np.savez(itmp, keys=np.array(keys), offsets=offs, lengths=lens)
    os.replace(tmp, emb_path)
    os.replace(itmp, idx_path)


def collate_captions(embs, pad_multiple=8, max_length=320, pad_to=None):
    """Pads real-token outputs to T = the longest caption rounded up to pad_multiple (at most max_length) or to a
    bucket edge: (emb [B, T, dim] bf16 with zeros after each caption, mask [B, T] bool, left-aligned)
    (reference gpic_dataset.py:662-685)."""
    lens = [int(e.shape[0]) for e in embs]
    T = pad_to or min(-(-max(lens) // pad_multiple) * pad_multiple, max_length)
    assert max(lens) <= T, (max(lens), T)
    out = torch.zeros(len(embs), T, embs[0].shape[1], dtype=torch.bfloat16)
    mask = torch.zeros(len(embs), T, dtype=torch.bool)
    for r, (e, n) in enumerate(zip(embs, lens)):
        out[r, :n] = e
        mask[r, :n] = True
    return out, mask


_BAD_MASKS = {}  # device -> int32 count of caption masks that were not left-aligned (checked on the host later)


def assert_left_aligned(mask):
    """Every mask row is a prefix of Trues (the attention kernels count a caption's keys from position 0).
    On the host it raises at once; on a GPU the check stays on the device (no sync, no device-side assert that would
    take the context down): violations are counted, and mask_errors() reports them at a log step."""
    n = mask.sum(1, keepdim=True)
    ok = (mask == (torch.arange(mask.shape[1], device=mask.device)[None] < n)).all()
    if mask.is_cuda:
        c = _BAD_MASKS.get(mask.device)
        if c is None:
            c = _BAD_MASKS[mask.device] = torch.zeros((), dtype=torch.int32, device=mask.device)
        c.add_((~ok).to(torch.int32))
    else:
        assert bool(ok), "caption masks must be left-aligned"


def mask_errors(device=None):
    """Host-side count of non-left-aligned caption masks seen on the device(s) so far (one sync)."""
    return sum(int(c.item()) for d, c in _BAD_MASKS.items() if device is None or d == torch.device(device))
