"""Sample rebalancing (parallel/rebalance.py): the deal, and the exchange on 2 gloo ranks (host tensors)."""
import os
import random
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nano_gpic_b200.parallel.rebalance import Rebalancer, deal


def test_deal_balances_and_keeps_counts():
    rng = random.Random(0)
    for world, B in [(2, 8), (4, 16), (8, 32)]:
        lens = [[rng.randint(8, 320) if r == 0 else rng.randint(8, 40) for _ in range(B)] for r in range(world)]
        dst = deal(lens, B)
        counts = [sum(dst[r][i] == d for r in range(world) for i in range(B)) for d in range(world)]
        assert counts == [B] * world
        load = [0] * world
        for r in range(world):
            for i in range(B):
                load[dst[r][i]] += lens[r][i]
        before = [sum(x) for x in lens]
        assert max(load) - min(load) <= max(max(x) for x in lens)
        assert max(load) < max(before)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, T, D = 8, 48, 4
    g = torch.Generator().manual_seed(rank)
    lens = torch.randint(30, 49, (B,), generator=g) if rank == 0 else torch.randint(1, 9, (B,), generator=g)
    ids = torch.arange(B) + 10 * rank
    img = ids.view(B, 1, 1, 1).expand(B, 4, 4, 3).to(torch.uint8).contiguous()
    mask = torch.arange(T)[None, :] < lens[:, None]
    cap = (ids.view(B, 1, 1).float() + 1).expand(B, T, D).to(torch.bfloat16) * mask[:, :, None]
    rb = Rebalancer(pad_multiple=8)
    img2, cap2, mask2 = rb(img, cap, mask)
    got = []
    for j in range(B):
        sid = int(img2[j, 0, 0, 0])
        n = int(mask2[j].sum())
        ok = bool((cap2[j, :n] == sid + 1).all()) and bool((cap2[j, n:] == 0).all())
        ok = ok and bool(mask2[j, :n].all())
        got.append((sid, n, ok))
    before, after = rb.last_loads
    out[rank] = (got, before, after, tuple(cap2.shape), cap2.dtype == torch.bfloat16)
    dist.destroy_process_group()


def test_exchange_two_ranks():
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _port(), out), nprocs=2, join=True)
    ids, lens = {}, {}
    for r in range(2):
        got, before, after, shape, bf16 = out[r]
        assert bf16 and shape[0] == 8 and shape[1] % 8 == 0
        for sid, n, ok in got:
            assert ok, (r, sid)
            ids[sid] = ids.get(sid, 0) + 1
            lens[sid] = n
    assert sorted(ids) == list(range(8)) + list(range(10, 18)) and set(ids.values()) == {1}
    before, after = out[0][1], out[0][2]
    assert max(after) < max(before)
