"""Collective microbenchmark on one node: this package's peer-memory kernels against NCCL for the two collectives of
the sharded (zero) data-parallel step, over bucket sizes of the ladder widths.

    torchrun --standalone --nproc-per-node N -m nano_gpic_b200.tools.bench_comm [--widths 768 1024 1792] [--iters 20]
    torchrun --standalone --nproc-per-node N -m nano_gpic_b200.tools.bench_comm --shapes [--widths ...]

reduce-scatter: an fp32 bucket of `W x seg` elements, every rank's segment summed over ranks (p2p: push into the
owners' receive slots + rank-ordered reduce, csrc/p2p.cu; nccl: reduce_scatter_tensor). weight broadcast / all-gather:
each owner's bf16 segment to every rank (p2p: the owner's fp32 master cast and stored into every rank's buffer; nccl:
all_gather_into_tensor of the bf16 segment). Bucket sizes: the matrices of one transformer block of width w
(24 w^2 parameters) times the blocks per 1000 MB bucket. Times are CUDA events around `iters` back-to-back calls,
the max over ranks; GB/s counts the bytes each rank sends over NVLink ((W - 1) / W of the bucket), compared with the
measured 770 GB/s per direction of a peer copy on this pool.

--shapes: the bucket is one weight matrix of each shape of the sweep, w x w, w x 3w, 3w x w and the SwiGLU halves
w x 4w, 4w x w, for each width. Besides the two collectives it times the Newton-Schulz orthogonalisation (5 quintic
steps on the tcgen05 GEMM, bf16) of that matrix, the work an owner does between them in the Muon step (gradient to
the owner, NS, bf16 update to every rank), and reports each stage against its roofline: bytes over NVLink at 770 GB/s
for the collectives, FLOPs at the measured bf16 GEMM peak for NS.
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
    ap.add_argument("--shapes", action="store_true", help="buckets of single matrices (w x w, w x 3w, 3w x w, w x 4w, "
                                                            "4w x w) and the Newton-Schulz step")
    a = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    W, rank = dist.get_world_size(), dist.get_rank()
    from ..parallel.ddp import P2PTransport
    rows = []
    cases = []
    for w in a.widths:
        if a.shapes:
            cases += [(w, (r, c)) for r, c in [(w, w), (w, 3 * w), (3 * w, w), (w, 4 * w), (4 * w, w)]]
        else:
            cases.append((w, None))
    for w, shape in cases:
        if shape is None:
            block = 24 * w * w
            per_bucket = max(1, (1000 * 1024 * 1024 // 4) // block)
            elems = block * per_bucket
        else:
            per_bucket, elems = 0, shape[0] * shape[1]
        seg = -(-elems // W) // 64 * 64
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
        row = {"width": w, "world": W, "bucket_params": n}
        if shape is None:
            row["blocks_per_bucket"] = per_bucket
        else:
            row["shape"] = list(shape)
            from ..optim.muon import msign
            from .bench_kernels import peaks
            g = torch.randn(1, *shape, device=dev)
            t_ns = timed(lambda: msign(g, steps=5), a.iters)
            r_, c_ = min(shape), max(shape)  # NS works on the wide orientation: X [r_, c_]
            fl = 5 * (2 * r_ * r_ * c_ + 2 * r_ ** 3 + 2 * r_ * r_ * c_)
            pk = peaks()[0]
            row["ns_us"] = round(t_ns * 1e6, 1)
            row["ns_tflops"] = round(fl / t_ns / 1e12, 1)
            row["ns_frac_of_bf16_peak"] = round(fl / t_ns / 1e12 / pk, 3)
        for k, v in t.items():
            gb = (W - 1) / W * n * sent[k] / 1e9
            row[k + "_us"] = round(v * 1e6, 1)
            row[k + "_GBps"] = round(gb / v, 1)
            row[k + "_frac_nvlink"] = round(gb / v / NVLINK_GBS, 3)
        if shape is not None:
            # the Muon step of one unit, stage by stage: gradient to the owner, NS there, the bf16 update to every rank
            row["muon_pipeline_p2p_us"] = round((t["p2p_reduce_scatter"] + t_ns + t["p2p_weight_broadcast"]) * 1e6, 1)
            row["muon_pipeline_nccl_us"] = round((t["nccl_reduce_scatter"] + t_ns + t["nccl_all_gather"]) * 1e6, 1)
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
