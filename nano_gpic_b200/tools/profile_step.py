"""Kernel-time breakdown of one training step (torch.profiler / CUPTI), grouped by kernel name.

    python -m nano_gpic_b200.tools.profile_step [--size d12] [--micro-batch 128] [--accum 1] [--out table.txt]

For analysis only: times under a profiler are not benchmark numbers (bench.py times without one).
"""
import argparse

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", default="d12")
    ap.add_argument("--micro-batch", type=int, default=128)
    ap.add_argument("--accum", type=int, default=1)
    ap.add_argument("--caption-len", type=int, default=128)
    ap.add_argument("--out", default=None)
    ap.add_argument("--rows", type=int, default=40)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    a = ap.parse_args()
    import sys, os
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    from bench import synthetic_batch
    from nano_gpic_b200.train.trainer import Trainer
    dev = torch.device("cuda", 0)
    gb = a.micro_batch * a.accum
    batch = synthetic_batch(gb, a.caption_len, 2048, seed=0, device=dev)
    if a.impl == "reference":  # the reference arm of bench.py, one step
        import types
        import bench
        ns = types.SimpleNamespace(size=a.size, micro_batch=a.micro_batch, global_batch=gb, caption_len=a.caption_len,
                                   warmup=3, steps=1, no_e2e=True)
        step = bench.reference_step_fn(ns, 0, 1, dev)
        run = lambda: step(*batch)
    else:
        tr = Trainer.for_ladder(a.size, device=dev, micro_batch=a.micro_batch, global_batch=gb)
        run = lambda: tr.train_step(*batch)
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        run()
        torch.cuda.synchronize()
    table = prof.key_averages().table(sort_by="cuda_time_total", row_limit=a.rows, max_name_column_width=90)
    print(table)
    tot = sum(e.device_time_total for e in prof.key_averages())
    print(f"total device time {tot / 1e3:.1f} ms for {gb} images")
    if a.out:
        with open(a.out, "w") as f:
            f.write(table + f"\ntotal device time {tot / 1e3:.1f} ms for {gb} images\n")


if __name__ == "__main__":
    main()
