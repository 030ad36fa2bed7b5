"""Shared caption-length buckets across ranks (reference baselines/PixelGen/src/data/shared_bucket_loader.py).

Every rank keeps a pool of ready batches per bucket (a bucket = a range of padded caption lengths, padded to its edge);
before each micro-batch the ranks all-reduce (MIN, on a gloo group) their pool sizes and take one batch from the bucket
every rank holds most of (ties to the shorter bucket), so every rank trains micro-batch k at the same caption length
and no rank waits for a longer one. A rank at pool_cap makes the micro-batch free: each rank takes its own fullest
bucket. The loader never ends: a finished pass of the wrapped iterable restarts inside the same iterator.
"""
import os
from collections import deque

import torch
import torch.distributed as dist

EDGES = (16, 24, 32, 40, 48, 56, 64, 144, 176, 320)


def choose(min_counts):
    """The bucket every rank holds most of (the first among ties), or None if no bucket is held by every rank."""
    best = max(range(len(min_counts)), key=lambda i: (min_counts[i], -i))
    return best if min_counts[best] > 0 else None


def bucket_of(length, edges=EDGES, pad_multiple=8, max_length=320):
    import bisect
    P = min(-(-length // pad_multiple) * pad_multiple, max_length)
    return bisect.bisect_left(edges, P)


class SharedBucketLoader:
    """loader yields (images, captions, meta) batches whose meta["text_mask"].shape[1] is a bucket edge."""

    def __init__(self, loader, edges=EDGES, pool_min=None, pool_cap=None, allreduce_min=None):
        self.loader, self.edges = loader, list(edges)
        self.pool_min = pool_min or 2 * len(self.edges)
        self.pool_cap = pool_cap or int(os.environ.get("GPIC_SHARED_BUCKET_POOL_CAP", "40"))
        self._allreduce_min = allreduce_min
        self.group = None
        self.taken = [0] * len(self.edges)
        self.passes = 0

    def __iter__(self):
        pools = [deque() for _ in self.edges]
        it = iter(self.loader)

        def pull():
            nonlocal it
            try:
                b = next(it)
            except StopIteration:
                self.passes += 1
                it = iter(self.loader)
                try:
                    b = next(it)
                except StopIteration:
                    raise RuntimeError("the training loader gave no batch in a whole data pass") from None
            pools[self.edges.index(b[2]["text_mask"].shape[1])].append(b)

        def min_counts(over):
            counts = [len(q) for q in pools] + [-1 if over else 0]
            if self._allreduce_min is not None:
                return self._allreduce_min(counts)
            if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
                return counts
            if self.group is None:
                self.group = dist.new_group(backend="gloo")
            t = torch.tensor(counts, dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.group)
            return t.tolist()

        started = False
        while True:
            over = sum(len(q) for q in pools) >= self.pool_cap
            if started and not over and sum(len(q) for q in pools) >= self.pool_min:
                pull()
            started = True
            while sum(len(q) for q in pools) < self.pool_min:
                pull()
            while True:
                mins = min_counts(over)
                if mins[-1] < 0:
                    b = max(range(len(pools)), key=lambda i: (len(pools[i]), -i))
                else:
                    b = choose(mins[:-1])
                if b is not None and pools[b]:
                    self.taken[b] += 1
                    yield pools[b].popleft()
                    break
                pull()
