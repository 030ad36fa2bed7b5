"""Data parallelism on 2 GPUs over NCCL: ddp and zero modes train the d12 architecture at reduced depth for a few steps
and must agree with each other (same data, same initial weights) within bf16 kernel noise; the collectives run on the
side stream under the backward. Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out, transport="nccl"):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from nano_gpic_b200.train.trainer import Trainer
        tr = Trainer.for_ladder("d12", device=dev, world=world, rank=rank, micro_batch=8, global_batch=32, dp=mode,
                                bucket_mb=40, model_kwargs={"num_blocks": 3, "num_text_blocks": 1},
                                transport=transport)
        g = torch.Generator().manual_seed(11)
        for s in range(3):
            img = torch.randint(0, 256, (32, 256, 256, 3), dtype=torch.uint8, generator=g)
            cap = torch.randn(32, 64, 2048, generator=g).bfloat16()
            mask = torch.arange(64)[None] < torch.randint(1, 65, (32,), generator=g)[:, None]
            t = torch.rand(32, generator=g)
            noise = torch.randn(32, 3, 256, 256, generator=g)
            sl = slice(rank * 16, (rank + 1) * 16)
            loss = tr.train_step(img[sl], cap[sl], mask[sl], t=t[sl], noise=noise[sl])
        torch.cuda.synchronize()
        from nano_gpic_b200.ops import status
        assert status.read() == 0
        tr.dp.gather_master()
        early = tr.dp.early
        if rank == 0:
            torch.save({"params": {n: p.detach().float().cpu() for n, p in tr.model.named_parameters()},
                        "loss": float(loss), "early": early, "buckets": len(tr.dp.layout.buckets)}, out)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ddp_and_zero_agree(tmp_path):
    res = {}
    for mode in ("ddp", "zero"):
        out = str(tmp_path / f"{mode}.pt")
        mp.spawn(_worker, args=(2, _port(), mode, out), nprocs=2, join=True)
        res[mode] = torch.load(out)
    a, b = res["ddp"], res["zero"]
    assert a["early"] >= 1 and b["early"] >= 1, (a["early"], b["early"])
    assert abs(a["loss"] - b["loss"]) < 1e-2 * abs(a["loss"]), (a["loss"], b["loss"])
    for n, p in a["params"].items():
        tol = 5e-2 if "adaLN_modulation.0.weight" in n else 1e-2
        err = float((p - b["params"][n]).norm() / (p.norm() + 1e-12))
        assert err < tol, (n, err)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_transport_matches_nccl(tmp_path):
    """zero mode over this package's peer-memory kernels (reduce-scatter, fused AdamW / Muon apply + weight broadcast)
    gives the NCCL transport's weights: the gradient sums are the same (2 ranks), the fused apply differs from torch's
    optimizer kernels only in fp32 rounding."""
    res = {}
    for tr in ("nccl", "p2p"):
        out = str(tmp_path / f"{tr}.pt")
        mp.spawn(_worker, args=(2, _port(), "zero", out, tr), nprocs=2, join=True)
        res[tr] = torch.load(out)
    # The zero-initialised adaLN weights take Muon updates of rank-deficient gradients: their trajectory amplifies
    # fp32 rounding differences (one process with another accumulation order moves them by tens of percent); every
    # other tensor must agree to 1e-4, and the losses closely.
    for n, p in res["nccl"]["params"].items():
        q = res["p2p"]["params"][n]
        err = float((p - q).norm() / (p.norm() + 1e-12))
        tol = 0.25 if "adaLN_modulation.0.weight" in n else (1e-3 if "adaLN_modulation" in n else 1e-4)
        assert err < tol, (n, err)
    assert abs(res["nccl"]["loss"] - res["p2p"]["loss"]) < 1e-3 * abs(res["nccl"]["loss"])
    assert res["p2p"]["early"] >= 1
