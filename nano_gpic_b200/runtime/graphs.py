"""CUDA-graph replay of a launch-bound function (the denoiser's forward in sampling).

A sampling step at a small batch is a few hundred short kernels, so the host's launch rate, not the GPU, sets its
time. `GraphedCall(fn)` records fn's kernels once per input signature (shapes, dtypes, device of its tensor
arguments) into a torch.cuda.CUDAGraph, after a warm-up on a side stream that builds every cached table and tensor
map; each later call copies the inputs into the graph's static buffers and replays it (one launch). Every tensor fn
reads must be an argument (anything it captures by closure is read at the captured address). The output is a fresh
tensor (a copy of the graph's static output), so results of earlier calls stay valid.

The reference samples eagerly (torch.compile'd denoiser, EulerSamplerJiT in
baselines/PixelGen/src/diffusion/flow_matching/sampling.py:114-201); CPU tensors run fn directly.
"""
import torch


class GraphedCall:
    def __init__(self, fn, warmup=2, max_graphs=16):
        self.fn, self.warmup, self.max_graphs = fn, warmup, max_graphs
        self.graphs = {}
        self.pool = None
        self.replays = 0

    @staticmethod
    def _key(args):
        return tuple((tuple(a.shape), a.dtype, str(a.device)) if torch.is_tensor(a) else ("const", a) for a in args)

    def _capture(self, args):
        static = [a.clone() if torch.is_tensor(a) else a for a in args]
        cur = torch.cuda.current_stream()
        side = torch.cuda.Stream()
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(self.warmup):
                self.fn(*static)
        cur.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(graph, pool=self.pool):
            out = self.fn(*static)
        return graph, static, out

    def __call__(self, *args):
        if not any(torch.is_tensor(a) and a.is_cuda for a in args) or torch.cuda.is_current_stream_capturing():
            return self.fn(*args)
        key = self._key(args)
        entry = self.graphs.get(key)
        if entry is None:
            if len(self.graphs) >= self.max_graphs:  # too many shapes: run eagerly instead of holding more pools
                return self.fn(*args)
            entry = self.graphs[key] = self._capture(args)
        graph, static, out = entry
        for s, a in zip(static, args):
            if torch.is_tensor(s):
                s.copy_(a)
        graph.replay()
        self.replays += 1
        return out.clone()
