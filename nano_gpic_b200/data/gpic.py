"""GPIC training data: webdataset tar shards with the cached text-encoder outputs.

Stages (reference baselines/PixelGen/src/data/dataset/gpic_dataset.py:402-866): shard order reshuffled at every pass
with Random(seed * 100003 + pass), rank r reading shards r, r + world, ... (EpochShuffledShards, :64-248; started
shards logged per rank so a resume skips them); samples with an image, a caption and a caption type; the caption's
cached encoder outputs attached; length grouping (windows of group_window samples sorted by caption length and cut
into batches, the batch order shuffled) or shared-bucket batches; then the image is decoded and random-cropped to 256
(uint8 HWC); the collate pads the captions (text_cache.collate_captions).
"""
import os
import random
import re
import time

import numpy as np
import torch
from torch.utils.data import DataLoader, IterableDataset, get_worker_info

from .augment import random_crop_arr
from .pil_resize import CropPlan, ResizeBatch, plan_random_crop
from .buckets import EDGES, bucket_of
from .tars import gpic_samples
from .text_cache import TextCache, collate_captions


def expand_pattern(pattern):
    """`dir/gpic_train_{00000..00800}.tar` -> the list of paths (zero-padded ranges, as webdataset's brace syntax)."""
    m = re.search(r"\{(\d+)\.\.(\d+)\}", pattern)
    if not m:
        return [pattern]
    a, b = m.group(1), m.group(2)
    w = len(a)
    return [pattern[:m.start()] + str(i).zfill(w) + pattern[m.end():] for i in range(int(a), int(b) + 1)]


def _rank_world():
    """(rank, world) from torch.distributed, else from RANK / WORLD_SIZE. A world of several ranks whose rank is not
    known is refused: taking rank 0 would make every rank read rank 0's shards."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world > 1 and "RANK" not in os.environ:
        raise RuntimeError(f"WORLD_SIZE={world} but no RANK and no torch.distributed group: the shard split is unknown")
    return int(os.environ.get("RANK", 0)), world


class EpochShuffledShards:
    """The shard order of every pass over the data, split over ranks, with a per-rank log of started shards that a
    resume reads: shards started before the stop are not read again in that pass (reference
    baselines/PixelGen/src/data/dataset/gpic_dataset.py:64-248).

    Pass p shuffles the urls with Random(seed * 100003 + p); rank r takes every world-th shard from position r. The log
    `shards_started_rank<r>.txt` gets one line `<time> <pass> <url>` when a shard starts. On construction the log gives
    the resume point: the newest pass that has a logged shard, minus its logged shards, or the next pass when all of
    this rank's shards of that pass were started. A torn last line (a worker killed inside its write) is dropped. A log
    that names a shard this rank would not read in that pass (another seed, shard list or number of ranks) is refused
    with ValueError rather than silently mixing two splits; so is a change of rank or world between construction and
    iteration."""

    def __init__(self, urls, seed, log_dir=None):
        self.urls, self.seed = list(urls), int(seed)
        self.rank, self.world = _rank_world()
        self.log_path = os.path.join(log_dir, f"shards_started_rank{self.rank}.txt") if log_dir else None
        self.passes, self.skip = self._resume_point() if self.log_path else (0, set())

    def check_rank(self):
        now = _rank_world()
        if now != (self.rank, self.world):
            raise ValueError(f"rank or world changed since the shard split was made: {now} != {(self.rank, self.world)}")

    def perm(self, p):
        urls = list(self.urls)
        random.Random(self.seed * 100003 + p).shuffle(urls)
        return urls

    def _resume_point(self):
        """(pass, shards started in it) from this rank's log; a torn last line is ignored."""
        if not os.path.exists(self.log_path):
            return 0, set()
        p, started = 0, set()
        with open(self.log_path) as f:
            for line in f:
                parts = line.split()
                if len(parts) != 3 or not line.endswith("\n"):
                    continue
                q = int(parts[1])
                if q > p:
                    p, started = q, set()
                if q == p:
                    started.add(parts[2])
        mine = set(self.perm(p)[self.rank::self.world])
        foreign = started - mine
        if foreign:
            raise ValueError(f"{self.log_path}: pass {p} logs {len(foreign)} shard(s) that rank {self.rank} of "
                             f"{self.world} does not read with seed {self.seed} (another seed, shard list or number "
                             f"of ranks?), e.g. {sorted(foreign)[0]}")
        if started == mine:
            return p + 1, set()
        return p, started

    def log_started(self, p, url):
        if self.log_path:
            with open(self.log_path, "a") as f:
                f.write(f"{time.time():.3f} {p} {url}\n")

    def shards_of_pass(self, p):
        mine = self.perm(p)[self.rank::self.world]
        if p == self.passes and self.skip:
            mine = [u for u in mine if u not in self.skip]
        return mine


class GPICDataset(IterableDataset):
    def __init__(self, tar_pattern, emb_dir, seed=0, image_size=256, group_window=1024, group_batch=128,
                 pad_multiple=8, text_max_length=320, shared_bucket=False, bucket_edges=EDGES, log_dir=None,
                 min_crop_frac=0.8, max_crop_frac=1.0, gpu_resize=None):
        super().__init__()
        # gpu_resize (reference lever C, GPIC_MFU_GPU_RESIZE): workers plan the region crop and the bicubic passes run
        # on the GPU for the whole batch (data/pil_resize.py), byte-identical to the crop done in Pillow
        if gpu_resize is None:
            gpu_resize = os.environ.get("GPIC_MFU_GPU_RESIZE", "0") == "1"
        self.gpu_resize = bool(gpu_resize)
        self.urls = expand_pattern(tar_pattern)
        self.emb_dir, self.seed, self.image_size = emb_dir, seed, image_size
        self.group_window, self.group_batch = group_window, group_batch
        self.pad_multiple, self.text_max_length = pad_multiple, text_max_length
        self.shared_bucket, self.bucket_edges = shared_bucket, tuple(bucket_edges)
        self.shards = EpochShuffledShards(self.urls, seed, log_dir)
        self.crop = (min_crop_frac, max_crop_frac)
        self._cache = None

    def _samples(self, p):
        wi = get_worker_info()
        self.shards.check_rank()
        shards = self.shards.shards_of_pass(p)
        if wi is not None:
            shards = shards[wi.id::wi.num_workers]
        if self._cache is None:
            self._cache = TextCache(self.emb_dir)
        for url in shards:
            self.shards.log_started(p, url)
            name = os.path.basename(url)[:-len(".tar")]
            for s in gpic_samples(url):
                s["text_emb"] = self._cache.read(name, s["key"])   # a sample without cached outputs stops the run
                s["text_len"] = int(s["text_emb"].shape[0])
                yield s

    def _grouped(self, src, rng):
        buf = []
        for s in src:
            buf.append(s)
            if len(buf) == self.group_window:
                yield from self._flush(buf, rng)
                buf = []
        if buf:
            yield from self._flush(buf, rng)

    def _flush(self, items, rng):
        items.sort(key=lambda s: s["text_len"])
        B = self.group_batch
        chunks = [items[i:i + B] for i in range(0, len(items) - B + 1, B)]
        rng.shuffle(chunks)
        for c in chunks:
            yield from c

    def _bucketed(self, src):
        queues = [[] for _ in self.bucket_edges]
        for s in src:
            q = bucket_of(s["text_len"], self.bucket_edges, self.pad_multiple, self.text_max_length)
            queues[q].append(s)
            if len(queues[q]) == self.group_batch:
                for x in queues[q]:
                    x["pad_to"] = self.bucket_edges[q]
                    yield x
                queues[q] = []

    def _finish(self, s, rng):
        import io
        from PIL import Image
        pil = Image.open(io.BytesIO(s["image"])).convert("RGB")
        if self.gpu_resize:
            img = plan_random_crop(pil, self.image_size, *self.crop, rng=rng)
        else:
            img = torch.from_numpy(np.asarray(random_crop_arr(pil, self.image_size, *self.crop, rng=rng), dtype=np.uint8))
        return (img, s["caption"],
                {"caption_type": s["caption_type"], "text_emb": s["text_emb"], "pad_to": s.get("pad_to")})

    def __iter__(self):
        wi = get_worker_info()
        rng = random.Random(self.seed * 1009 + (wi.id if wi else 0))
        p = self.shards.passes
        src = self._samples(p)
        src = self._bucketed(src) if self.shared_bucket else self._grouped(src, rng)
        last, repeats = None, 0
        for s in src:
            try:
                out = self._finish(s, rng)
                last, repeats = out, 0
            except Exception:
                repeats += 1
                if last is None or repeats > 8:
                    raise
                out = last   # an image that fails to decode repeats the sample before it
            yield out

    def collate(self, samples):
        if isinstance(samples[0][0], CropPlan):  # GPU resize: the batch's crops run on the device (ResizeBatch.run)
            imgs = ResizeBatch([s[0] for s in samples], self.image_size)
        else:
            imgs = torch.stack([s[0] for s in samples])
        emb, mask = collate_captions([s[2]["text_emb"] for s in samples], self.pad_multiple, self.text_max_length,
                                     pad_to=samples[0][2].get("pad_to"))
        return imgs, [s[1] for s in samples], {"caption_type": [s[2]["caption_type"] for s in samples],
                                               "text_emb": emb, "text_mask": mask}

    def build_dataloader(self, batch_size, num_workers=8):
        return DataLoader(self, batch_size=batch_size, num_workers=num_workers, collate_fn=self.collate,
                          persistent_workers=num_workers > 0, pin_memory=True, drop_last=True)


class SyntheticGPIC:
    """Synthetic batches of the benchmark's shape: uint8 images uniform (x uniform in [-1, 1]), N(0, 1) caption
    features, left-aligned masks with lengths uniform in [1, T]. Batch i is drawn from a generator seeded
    (seed * 1000003 + i), so a loader started at `start` (a resume) yields the batches an uninterrupted run would."""

    def __init__(self, batch, T=128, D=2048, image_size=256, seed=0, start=0):
        self.batch, self.T, self.D, self.size = batch, T, D, image_size
        self.seed, self.index = seed, start

    def __iter__(self):
        return self

    def __next__(self):
        g = torch.Generator().manual_seed(self.seed * 1000003 + self.index)
        self.index += 1
        B, T = self.batch, self.T
        img = torch.randint(0, 256, (B, self.size, self.size, 3), dtype=torch.uint8, generator=g)
        cap = torch.randn(B, T, self.D, generator=g).to(torch.bfloat16)
        lens = torch.randint(1, T + 1, (B,), generator=g)
        lens[0] = T
        mask = torch.arange(T)[None] < lens[:, None]
        return img, [""] * B, {"caption_type": ["synthetic"] * B, "text_emb": cap, "text_mask": mask}


class GPICWebDataset(GPICDataset):
    """GPICDataset under the reference's constructor (baselines/PixelGen/src/data/dataset/gpic_dataset.py:402-440
    init args), so its YAML `data.train_dataset` nodes build this loader: tar_dir + tar_pattern, the text-cache
    directory, length grouping (group_text_len, group_window) or shared buckets, caption padding. Arguments that only
    select the reference's alternative paths (shuffle_buffer, corrupted_csv, output_fields, is_val) are accepted."""

    def __init__(self, tar_dir, tar_pattern, emb_dir=None, shuffle_buffer=100, group_text_len=True, group_window=1024,
                 text_max_length=320, pad_multiple=8, shared_bucket=False, corrupted_csv=None, output_fields=None,
                 is_val=False, seed=None, batch_size=128, image_size=256, log_dir=None):
        seed = int(os.environ.get("GPIC_SHARD_SEED", 0)) if seed is None else seed
        if log_dir is None and not is_val:
            log_dir = os.environ.get("GPIC_SHARD_LOG_DIR")
        super().__init__(os.path.join(tar_dir, tar_pattern), emb_dir, seed=seed, image_size=image_size,
                         group_window=group_window if group_text_len else batch_size, group_batch=batch_size,
                         pad_multiple=pad_multiple, text_max_length=text_max_length, shared_bucket=shared_bucket,
                         log_dir=None if is_val else log_dir)  # only the training set keeps a shard log
        self.is_val = is_val


def gpic_jsonl_save_fn(image, metadata, root_path):
    """One HWC uint8 array -> <root>/<caption_type>_<key>.png."""
    from PIL import Image
    Image.fromarray(image).save(os.path.join(root_path, f"{metadata['caption_type']}_{metadata['key']}.png"))


class GPICJsonlDataset(torch.utils.data.Dataset):
    """Prediction prompts from a JSONL file of {key, caption, caption_type} records; each prompt is sampled
    num_samples_per_instance times, sample i starting from randn(latent_shape) of a CPU generator seeded i, the same
    noise for every prompt (reference baselines/PixelGen/src/data/dataset/gpic_jsonl_dataset.py:25-69)."""

    def __init__(self, jsonl_path, num_samples_per_instance=1, latent_shape=(3, 256, 256)):
        import json
        with open(jsonl_path) as f:
            self.records = [json.loads(line) for line in f if line.strip()]
        self.num_samples_per_instance = num_samples_per_instance
        self.latent_shape = list(latent_shape)

    def __len__(self):
        return len(self.records) * self.num_samples_per_instance

    def __getitem__(self, idx):
        rec = self.records[idx // self.num_samples_per_instance]
        sample = idx % self.num_samples_per_instance
        noise = torch.randn(self.latent_shape, generator=torch.Generator().manual_seed(sample), dtype=torch.float32)
        meta = {"key": rec["key"], "caption": rec["caption"], "caption_type": rec["caption_type"], "seed": sample,
                "save_fn": gpic_jsonl_save_fn}
        return noise, rec["caption"], meta
