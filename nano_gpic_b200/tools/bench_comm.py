"""Collective microbenchmark on one node: this package's peer-memory kernels against NCCL for the two collectives of
the sharded (zero) data-parallel step, over bucket sizes of the ladder widths.

    torchrun --standalone --nproc-per-node N -m nano_gpic_b200.tools.bench_comm [--widths 768 1024 1792] [--iters 20]

reduce-scatter: an fp32 bucket of `W x seg` elements, every rank's segment summed over ranks (p2p: push into the
owners' receive slots + rank-ordered reduce, csrc/p2p.cu; nccl: reduce_scatter_tensor). weight broadcast / all-gather:
each owner's bf16 segment to every rank (p2p: the owner's fp32 master cast and stored into every rank's buffer; nccl:
all_gather_into_tensor of the bf16 segment). Bucket sizes: the matrices of one transformer block of width w
(24 w^2 parameters) times the blocks per 1000 MB bucket. Times are CUDA events around `iters` back-to-back calls,
the max over ranks; GB/s counts the bytes each rank sends over NVLink ((W - 1) / W of the bucket), compared with the
measured 770 GB/s per direction of a peer copy on this pool.
"""
import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def timed(fn, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters * 1e-3], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--widths", type=int, nargs="+", default=[768, 1024, 1280, 1536, 1792])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    W, rank = dist.get_world_size(), dist.get_rank()
    from ..parallel.ddp import P2PTransport
    rows = []
    for w in a.widths:
        block = 24 * w * w
        per_bucket = max(1, (1000 * 1024 * 1024 // 4) // block)
        seg = -(-block * per_bucket // W) // 64 * 64
        n = seg * W
        tr = P2PTransport(n, 1, dev)
        tr.grad.normal_()
        master = torch.randn(n, device=dev)
        ref = tr.grad.clone()
        epoch = [0]   # reduce-scatter flags / acks
        wepoch = [0]  # weight-broadcast flags (their own channel)

        def p2p_rs():
            epoch[0] += 1
            tr.reduce_scatter(0, 0, seg, epoch[0])

        def p2p_bc():
            wepoch[0] += 1
            tr.broadcast_weights(master, 0, rank * seg, seg, wepoch[0])
            tr.wait_weights(0, 1, wepoch[0])

        def nccl_rs():
            dist.reduce_scatter_tensor(ref[rank * seg:(rank + 1) * seg], ref, op=dist.ReduceOp.SUM)

        w16 = torch.empty(n, dtype=torch.bfloat16, device=dev)

        def nccl_ag():
            dist.all_gather_into_tensor(w16, w16[rank * seg:(rank + 1) * seg])

        t = {"p2p_reduce_scatter": timed(p2p_rs, a.iters), "nccl_reduce_scatter": timed(nccl_rs, a.iters)}
        t["p2p_weight_broadcast"] = timed(p2p_bc, a.iters)
        t["nccl_all_gather"] = timed(nccl_ag, a.iters)
        sent = {"p2p_reduce_scatter": 4, "nccl_reduce_scatter": 4, "p2p_weight_broadcast": 2, "nccl_all_gather": 2}
        row = {"width": w, "world": W, "bucket_params": n, "blocks_per_bucket": per_bucket}
        for k, v in t.items():
            gb = (W - 1) / W * n * sent[k] / 1e9
            row[k + "_us"] = round(v * 1e6, 1)
            row[k + "_GBps"] = round(gb / v, 1)
            row[k + "_frac_nvlink"] = round(gb / v / NVLINK_GBS, 3)
        # correctness: the p2p segment equals the NCCL segment (fresh inputs, one call each)
        tr.grad.copy_(torch.randn(n, device=dev, generator=torch.Generator(dev).manual_seed(rank)))
        ref.copy_(tr.grad)
        epoch[0] += 1
        tr.reduce_scatter(0, 0, seg, epoch[0])
        nccl_rs()
        torch.cuda.synchronize()
        row["max_abs_diff_vs_nccl"] = float((tr.grad[rank * seg:(rank + 1) * seg] - ref[rank * seg:(rank + 1) * seg])
                                            .abs().max())
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
        tr.close()
        del tr
        torch.cuda.empty_cache()
    from ..ops import status
    status.check()
    if rank == 0 and a.json:
        with open(a.json, "w") as f:
            json.dump(rows, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
