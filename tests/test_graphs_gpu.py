"""CUDA-graph replay of the denoiser's forward (runtime/graphs.py): the replayed forward equals the eager one for new
inputs in the captured buffers, one graph per input signature, and a full Euler sampling run through it matches the
eager run."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _net():
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    torch.manual_seed(0)
    net = JiT_T2I(input_size=64, in_channels=3, num_groups=4, hidden_size=256, num_blocks=2, num_text_blocks=1,
                  patch_size=16, txt_embed_dim=64, txt_max_length=16).cuda().eval()
    with torch.no_grad():
        for p in net.parameters():
            p.add_(torch.randn_like(p) * 0.02)
    return net


def _inputs(B, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, 3, 64, 64, device="cuda", generator=g)
    t = torch.rand(B, device="cuda", generator=g)
    y = torch.randn(B, 16, 64, device="cuda", generator=g).bfloat16()
    m = torch.arange(16, device="cuda")[None] < torch.randint(1, 17, (B, 1), device="cuda", generator=g)
    return x, t, y, m


def test_graphed_forward_matches_eager():
    from nano_gpic_b200.runtime.graphs import GraphedCall
    net = _net()
    fn = lambda x, t, y, m: net(x, t, y, y_mask=m)
    gc = GraphedCall(fn)
    with torch.no_grad():
        for seed, B in ((1, 4), (2, 4), (3, 2), (4, 4)):
            args = _inputs(B, seed)
            assert torch.equal(gc(*args), fn(*args)), (seed, B)
    assert len(gc.graphs) == 2 and gc.replays == 4


def test_graphed_sampling_matches_eager():
    from nano_gpic_b200.diffusion.sampling import EulerSamplerJiT
    from nano_gpic_b200.runtime.graphs import GraphedCall
    net = _net()
    x, _, y, m = _inputs(2, 7)
    uncond = torch.zeros_like(y)
    null = torch.zeros_like(m)
    null[:, 0] = True
    sampler = EulerSamplerJiT(num_steps=6, guidance=2.0)
    outs = []
    for graphed in (False, True):
        call = GraphedCall(lambda a, b, c, d: net(a, b, c, y_mask=d)) if graphed else \
            (lambda a, b, c, d: net(a, b, c, y_mask=d))
        f = lambda a, b, c: call(a, b, c, torch.cat([null, m]) if c.shape[0] == 2 * m.shape[0] else m)
        outs.append(sampler(f, x, y, uncond))
    assert torch.equal(outs[0], outs[1])
