"""GraphedCall on CPU tensors runs the function directly (no CUDA graph)."""
import torch


def test_graphed_call_cpu_passthrough():
    from nano_gpic_b200.runtime.graphs import GraphedCall
    gc = GraphedCall(lambda a, b: a * 2 + b)
    a, b = torch.ones(3), torch.arange(3.0)
    assert torch.equal(gc(a, b), a * 2 + b) and not gc.graphs and gc.replays == 0
