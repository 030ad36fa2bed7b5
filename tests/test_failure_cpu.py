"""Failure detection on the host (no GPU involved): a rank that leaves between steps, with nothing in flight, and
never joins the next collective. The surviving rank's next collective must end with an error within the process
group's short timeout instead of waiting for good; the launcher then decides what to do (the job scripts exit and
resume from the last checkpoint)."""
import datetime
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)  # a healthy step on both ranks
    if rank == 1:
        out[1] = "left"
        os._exit(0)  # leaves between steps and never joins the next collective
    t0 = time.time()
    try:
        dist.all_reduce(t)
        out[0] = "no error"
    except Exception as e:  # gloo reports the lost peer (closed connection or timeout)
        out[0] = f"error {type(e).__name__} after {time.time() - t0:.1f} s"
    os._exit(0)  # the peer is gone: no destroy_process_group


def test_lost_rank_ends_the_next_collective_with_an_error():
    out = mp.Manager().dict()
    t0 = time.time()
    mp.spawn(_worker, args=(_port(), out), nprocs=2, join=True)
    assert out[1] == "left"
    assert out[0].startswith("error"), out[0]
    assert time.time() - t0 < 60
