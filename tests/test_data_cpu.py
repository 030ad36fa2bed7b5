"""The data path on CPU: the per-rank shard log and its resume (modelled on the reference's
tools/test_shard_resume.py:62-208), the shared caption-length buckets with an injected MIN all-reduce (as the
reference's SharedBucketLoader test hook, shared_bucket_loader.py:51-56,96-141), and GPICWebDataset end to end on
synthetic tar shards with a text cache."""
import io
import json
import os
import random
import tarfile
import threading

import numpy as np
import pytest
import torch

from nano_gpic_b200.data import gpic as G
from nano_gpic_b200.data.buckets import EDGES, SharedBucketLoader, bucket_of
from nano_gpic_b200.data.text_cache import write_shard

URLS = [f"/d/gpic_train_{i:05d}.tar" for i in range(64)]
SEED, WORLD = 20261106, 8


@pytest.fixture
def as_rank(monkeypatch):
    def set_rank(r, world=WORLD):
        monkeypatch.setenv("RANK", str(r))
        monkeypatch.setenv("WORLD_SIZE", str(world))
    return set_rank


def _log(d, r, rows, torn=None):
    with open(os.path.join(d, f"shards_started_rank{r}.txt"), "a") as f:
        f.writelines(f"{100 + i}.000 {p} {u}\n" for i, (p, u) in enumerate(rows))
        if torn:
            f.write(torn)


def test_node_split_covers_every_shard_once(as_rank):
    seen = []
    for r in range(WORLD):
        as_rank(r)
        s = G.EpochShuffledShards(URLS, SEED)
        mine = s.shards_of_pass(0)
        assert mine == s.perm(0)[r::WORLD]
        seen += mine
    assert sorted(seen) == sorted(URLS)
    as_rank(0)
    s = G.EpochShuffledShards(URLS, SEED)
    assert s.perm(0) != s.perm(1) and sorted(s.perm(1)) == sorted(URLS)  # reshuffled every pass


def test_resume_skips_started_shards(tmp_path, as_rank):
    """A stopped launch logged some shards (also the one in progress); the resume reads the rest of this rank's pass
    once, and the next pass is whole."""
    d = str(tmp_path)
    r = 3
    as_rank(r)
    s = G.EpochShuffledShards(URLS, SEED, d)
    mine = s.shards_of_pass(0)
    for u in mine[:3]:  # the dataset logs a shard when it starts it
        s.log_started(0, u)
    again = G.EpochShuffledShards(URLS, SEED, d)
    assert (again.passes, again.skip) == (0, set(mine[:3]))
    rest = again.shards_of_pass(0)
    assert rest == mine[3:] and sorted(rest + mine[:3]) == sorted(mine)
    assert again.shards_of_pass(1) == again.perm(1)[r::WORLD]


def test_whole_pass_logged_resumes_in_the_next(tmp_path, as_rank):
    d = str(tmp_path)
    r = 5
    as_rank(r)
    s = G.EpochShuffledShards(URLS, SEED)
    mine0, mine1 = s.perm(0)[r::WORLD], s.perm(1)[r::WORLD]
    _log(d, r, [(0, u) for u in mine0])
    c = G.EpochShuffledShards(URLS, SEED, d)
    assert (c.passes, c.skip) == (1, set())
    _log(d, r, [(1, u) for u in mine1[:2]])
    c = G.EpochShuffledShards(URLS, SEED, d)
    assert (c.passes, c.skip) == (1, set(mine1[:2])) and c.shards_of_pass(1) == mine1[2:]


def test_foreign_log_is_refused(tmp_path, as_rank):
    """A log written with another seed names shards this rank does not read: the resume stops."""
    d = str(tmp_path)
    r = 1
    as_rank(r)
    mine = G.EpochShuffledShards(URLS, SEED).perm(0)[r::WORLD]
    other = G.EpochShuffledShards(URLS, SEED + 1).perm(0)[r::WORLD]
    foreign = next(u for u in other if u not in mine)
    _log(d, r, [(0, foreign)])
    with pytest.raises(ValueError, match="does not read"):
        G.EpochShuffledShards(URLS, SEED, d)


def test_torn_last_line_is_dropped(tmp_path, as_rank):
    d = str(tmp_path)
    r = 2
    as_rank(r)
    mine = G.EpochShuffledShards(URLS, SEED).perm(0)[r::WORLD]
    _log(d, r, [(0, u) for u in mine[:3]], torn="104.000 0")
    c = G.EpochShuffledShards(URLS, SEED, d)
    assert (c.passes, c.skip) == (0, set(mine[:3]))


def test_unknown_rank_is_refused(monkeypatch):
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.setenv("WORLD_SIZE", "8")
    with pytest.raises(RuntimeError, match="no RANK"):
        G.EpochShuffledShards(URLS, SEED)


def test_rank_change_is_refused(as_rank):
    as_rank(1)
    s = G.EpochShuffledShards(URLS, SEED)
    as_rank(2)
    with pytest.raises(ValueError, match="changed"):
        s.check_rank()


def test_only_the_training_set_logs(tmp_path, monkeypatch, as_rank):
    as_rank(0, 1)
    monkeypatch.setenv("GPIC_SHARD_LOG_DIR", str(tmp_path))
    tr = G.GPICWebDataset(tar_dir="/nonexistent", tar_pattern="x_{00000..00003}.tar")
    va = G.GPICWebDataset(tar_dir="/nonexistent", tar_pattern="x_{00000..00003}.tar", is_val=True)
    assert tr.shards.log_path == os.path.join(str(tmp_path), "shards_started_rank0.txt")
    assert va.shards.log_path is None


# ----------------------------------------------------------------------------------------------- shared buckets
class _FakeLoader:
    """Batches of one bucket each (meta text_mask of the bucket's edge), lengths drawn per rank."""

    def __init__(self, seed, n=400):
        self.seed, self.n = seed, n

    def __iter__(self):
        rng = random.Random(self.seed)
        for i in range(self.n):
            e = rng.choice(EDGES[:7]) if rng.random() < 0.85 else rng.choice(EDGES[7:])
            yield (torch.tensor([i]), ["c"], {"text_mask": torch.ones(1, e, dtype=torch.bool)})


class _MinAllReduce:
    """An all-reduce MIN between threads standing in for ranks (the loader's allreduce_min hook)."""

    def __init__(self, world):
        self.world, self.barrier = world, threading.Barrier(world)
        self.slots = [None] * world
        self.calls = [0] * world

    def for_rank(self, r):
        def reduce(counts):
            self.slots[r] = list(counts)
            self.calls[r] += 1
            self.barrier.wait()
            out = [min(c) for c in zip(*self.slots)]
            self.barrier.wait()
            return out
        return reduce


def test_shared_buckets_agree_across_ranks():
    """Every rank trains micro-batch k at the same caption length, except for free steps when a pool is over its cap;
    no rank waits for a bucket it lacks; the pools stay bounded."""
    world, steps = 3, 150
    red = _MinAllReduce(world)
    picks = [[] for _ in range(world)]
    loaders = [SharedBucketLoader(_FakeLoader(10 + r), pool_cap=24, allreduce_min=red.for_rank(r)) for r in range(world)]

    def run(r):
        it = iter(loaders[r])
        for _ in range(steps):
            b = next(it)
            picks[r].append(b[2]["text_mask"].shape[1])
    ths = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in ths:
        t.start()
    for t in ths:
        t.join(timeout=60)
    assert all(len(p) == steps for p in picks)
    same = sum(len({picks[r][k] for r in range(world)}) == 1 for k in range(steps))
    assert same >= 0.8 * steps, same  # free steps (a rank over its cap) are the only disagreements
    assert sum(l.taken[i] for l in loaders for i in range(len(EDGES))) == world * steps
    assert bucket_of(17) == EDGES.index(24) and bucket_of(300) == EDGES.index(320) and bucket_of(1) == 0


# ----------------------------------------------------------------------------------- dataset on synthetic tars
def _jpeg(rng, w, h):
    from PIL import Image
    arr = (np.random.RandomState(rng.randrange(1 << 30)).rand(h, w, 3) * 255).astype(np.uint8)
    buf = io.BytesIO()
    Image.fromarray(arr).save(buf, format="JPEG")
    return buf.getvalue()


def _write_tar(path, samples):
    with tarfile.open(path, "w") as tar:
        for key, files in samples:
            for ext, data in files.items():
                ti = tarfile.TarInfo(f"{key}.{ext}")
                ti.size = len(data)
                tar.addfile(ti, io.BytesIO(data))


def test_gpic_web_dataset_on_synthetic_tars(tmp_path, as_rank):
    """Samples with an image, caption and caption type come out cropped to 64x64 uint8 with their cached caption
    features, grouped by caption length, padded per batch to a multiple of 8; samples without a caption are skipped;
    the shard log records each started shard."""
    as_rank(0, 1)
    rng = random.Random(0)
    tars, emb = tmp_path / "tars", tmp_path / "emb"
    tars.mkdir()
    cache = {}
    for s in range(2):
        samples, keys, embs = [], [], []
        for i in range(12):
            key = f"s{s}_{i:03d}"
            meta = {"caption": f"caption {key}", "caption_type": "short"}
            if i == 5:
                meta.pop("caption")  # filtered out like the training pipeline does
            samples.append((key, {"jpg": _jpeg(rng, 80 + i, 72), "json": json.dumps(meta).encode()}))
            n = rng.randint(1, 30)
            e = torch.randn(n, 2048).bfloat16()
            keys.append(key)
            embs.append(e)
            cache[key] = e
        _write_tar(str(tars / f"gpic_train_{s:05d}.tar"), samples)
        write_shard(str(emb), f"gpic_train_{s:05d}", keys, embs)
    ds = G.GPICWebDataset(tar_dir=str(tars), tar_pattern="gpic_train_{00000..00001}.tar", emb_dir=str(emb),
                          group_window=8, batch_size=4, image_size=64, log_dir=str(tmp_path), seed=3)
    loader = ds.build_dataloader(4, num_workers=0)
    batches = list(loader)
    assert len(batches) >= 4
    seen = 0
    for imgs, caps, meta in batches:
        assert imgs.shape == (4, 64, 64, 3) and imgs.dtype == torch.uint8
        y, m = meta["text_emb"], meta["text_mask"]
        lens = m.sum(1).tolist()
        assert y.shape[1] == -(-max(lens) // 8) * 8 and y.dtype == torch.bfloat16
        for r, c in enumerate(caps):
            key = c.split()[-1]
            assert torch.equal(y[r, :lens[r]], cache[key]) and not y[r, lens[r]:].any()
            assert key[-3:] != "005"
        assert max(lens) - min(lens) <= 30
        seen += 4
    with open(tmp_path / "shards_started_rank0.txt") as f:
        logged = [line.split()[2] for line in f]
    assert sorted(os.path.basename(u) for u in logged) == ["gpic_train_00000.tar", "gpic_train_00001.tar"]
    # a resume of the finished pass starts the next one
    again = G.EpochShuffledShards(ds.urls, 3, str(tmp_path))
    assert (again.passes, again.skip) == (1, set())
