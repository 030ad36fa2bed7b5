"""Data-parallel gradient reduction over the flat gradient buffer.

mode "nccl" (the baseline, as the reference's DDP: fp32 all-reduce of all gradients, averaged; reference
baselines/PixelGen/configs_h100/lite_ladder.yaml:7-12): one torch.distributed all-reduce per bucket of the flat buffer
(buckets on parameter boundaries, default 1000 MB like the reference's bucket_cap_mb).
"""
import torch
import torch.distributed as dist


class GradReducer:
    def __init__(self, flat, mode="nccl", bucket_mb=1000, group=None):
        self.flat = flat
        self.mode = mode
        self.group = group
        self.world = dist.get_world_size(group)
        self.buckets = flat.ranges(bucket_mb * 1024 * 1024 // 4)

    @torch.no_grad()
    def reduce(self):
        g = self.flat.grad
        for a, b in self.buckets:
            dist.all_reduce(g[a:b], op=dist.ReduceOp.SUM, group=self.group)
        g.mul_(1.0 / self.world)

    @torch.no_grad()
    def broadcast_params(self, src=0):
        dist.broadcast(self.flat.data, src, group=self.group)
        self.flat.sync_bf16()
