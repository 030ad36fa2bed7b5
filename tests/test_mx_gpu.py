"""MXFP8 quantization (csrc/mx.cu) and the block-scaled tcgen05 GEMM (csrc/gemm.cu, MX tiles).

The CUDA quantizer must match the PyTorch restatement bit for bit (values and scale bytes); the GEMMs are compared with
an fp32 PyTorch GEMM of the dequantized operands, followed by the same epilogue."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(a, b, rtol=1e-2, atol=1e-2):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= atol + rtol * ref, f"max err {err} vs ref max {ref}"


def _input(R, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(R, K, device="cuda", generator=g)
    # blocks of very different magnitude, an all-zero block and an all-zero row
    x = x * torch.pow(10.0, torch.randint(-3, 3, (R, K // 32, 1), device="cuda", generator=g).float()).repeat_interleave(
        32, 1).view(R, K)
    x[0, 32:64] = 0
    if R > 5:
        x[5] = 0
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("R,K", [(1, 128), (300, 384), (4096, 1024), (257, 4096)])
def test_quant_matches_torch(R, K):
    from nano_gpic_b200.ops import mx
    x = _input(R, K, seed=R + K)
    got = mx.quant(x)
    ref = mx._quant_torch(x.cpu())
    assert torch.equal(got.sf.cpu(), ref.sf), "scale bytes differ"
    assert torch.equal(got.q.cpu(), ref.q), "e4m3 values differ"
    # quantization error: at most half an e4m3 step (2^-4 relative to the block's power of two scale) per value
    deq = got.dequant().cpu()
    blk_max = x.float().cpu().view(R, K // 32, 32).abs().amax(-1, keepdim=True)
    err = (deq.view(R, K // 32, 32) - x.float().cpu().view(R, K // 32, 32)).abs()
    assert (err <= blk_max * 2.0 ** -4 + 1e-30).all()


def _operands(M, N, K, seed=0):
    from nano_gpic_b200.ops import mx
    torch.manual_seed(seed)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    xq, wq = mx.quant(x), mx.quant(w)
    return xq, wq, xq.dequant(), wq.dequant()


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (300, 640, 384), (4096, 4096, 1024), (77, 136, 256)])
def test_mx_linear(M, N, K):
    from nano_gpic_b200.ops import mx, status
    xq, wq, xd, wd = _operands(M, N, K)
    b = torch.randn(N, device="cuda")
    y = mx.linear(xq, wq, b)
    _close(y, xd @ wd.t() + b)
    torch.cuda.synchronize()
    assert status.read() == 0


@pytest.mark.parametrize("M,N,K", [(512, 1024, 1024), (300, 640, 4096)])
def test_mx_gated_residual(M, N, K):
    from nano_gpic_b200.ops import mx
    xq, wq, xd, wd = _operands(M, N, K, seed=1)
    rpg = 128
    G = (M + rpg - 1) // rpg
    res = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    gate_full = torch.randn(G, 3 * N, device="cuda").to(torch.bfloat16)
    gate = gate_full[:, N:2 * N]
    b = torch.randn(N, device="cuda")
    out, y = mx.linear_gated_residual(xq, wq, b, res, gate, rpg)
    yr = (xd @ wd.t() + b).to(torch.bfloat16)
    _close(y, yr)
    g = gate.float().repeat_interleave(rpg, 0)[:M]
    _close(out, res.float() + g * yr.float())


@pytest.mark.parametrize("M,H,K", [(4096, 4096, 1024), (300, 384, 256)])
def test_mx_swiglu(M, H, K):
    from nano_gpic_b200.ops import mx
    xq, wq, xd, wd = _operands(M, 2 * H, K, seed=2)
    act, pre = mx.swiglu_linear(xq, wq)
    pr = (xd @ wd.t()).to(torch.bfloat16)
    _close(pre, pr)
    x1, x2 = pr.float().chunk(2, dim=-1)
    _close(act, torch.nn.functional.silu(x1).to(torch.bfloat16).float() * x2)


def test_model_fp8_close_to_bf16():
    """d-small JiT-T2I: the MXFP8 forward's loss and gradients stay close to the bf16 ones."""
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    torch.manual_seed(0)
    net = JiT_T2I(input_size=64, in_channels=3, num_groups=4, hidden_size=256, num_blocks=2, num_text_blocks=1,
                  patch_size=16, txt_embed_dim=2048, txt_max_length=32).cuda()
    B = 4
    x = torch.randn(B, 3, 64, 64, device="cuda")
    t = torch.rand(B, device="cuda")
    y = torch.randn(B, 32, 2048, device="cuda").to(torch.bfloat16)
    m = torch.ones(B, 32, dtype=torch.bool, device="cuda")
    m[:, 20:] = False
    with torch.no_grad():  # the zero-initialised output and gate layers would make every output 0
        for prm in net.parameters():
            prm.add_(torch.randn_like(prm) * 0.02)
    outs, grads = [], []
    for mode in (None, "mx"):
        net.set_fp8(mode)
        net.zero_grad(set_to_none=True)
        o = net(x, t, y, y_mask=m)
        o.float().square().mean().backward()
        outs.append(o.float())
        grads.append(net.blocks[0].mlp.w12.weight.grad.clone())
    rel = (outs[1] - outs[0]).norm() / outs[0].norm()
    assert rel < 0.05, rel
    relg = (grads[1] - grads[0]).norm() / grads[0].norm()
    assert relg < 0.1, relg


@pytest.mark.parametrize("M,C,mod", [(512, 1024, True), (300, 384, True), (256, 768, False)])
def test_norm_with_mx_output_equals_separate_quant(M, C, mod):
    """The norm kernel's MXFP8 copy of h equals quantizing its bf16 output separately, byte for byte."""
    from nano_gpic_b200.ops import mx, norm
    torch.manual_seed(3)
    x = torch.randn(M, C, device="cuda").to(torch.bfloat16)
    w = torch.rand(C, device="cuda") + 0.5
    G = (M + 127) // 128
    sh = (torch.randn(G, C, device="cuda") * 0.1).to(torch.bfloat16) if mod else None
    sc = (torch.randn(G, C, device="cuda") * 0.1).to(torch.bfloat16) if mod else None
    h, r = norm.rms_mod_fwd(x, w, sh, sc, 128)
    h2, r2, hq = norm.rms_mod_fwd_mx(x, w, sh, sc, 128)
    ref = mx.quant(h)
    assert torch.equal(h, h2) and torch.equal(r, r2)
    assert torch.equal(hq.q, ref.q)
    assert torch.equal(hq.sf, ref.sf)


@pytest.mark.parametrize("M,H,K", [(4096, 4096, 1024), (300, 384, 256)])
def test_mx_swiglu_act_output_equals_separate_quant(M, H, K):
    """The SwiGLU epilogue's MXFP8 copy of act equals quantizing its bf16 act separately, byte for byte."""
    from nano_gpic_b200.ops import mx
    xq, wq, _, _ = _operands(M, 2 * H, K, seed=4)
    act, pre, aq = mx.swiglu_linear(xq, wq, quant_act=True)
    act2, pre2 = mx.swiglu_linear(xq, wq)
    assert torch.equal(act, act2) and torch.equal(pre, pre2)
    ref = mx.quant(act)
    assert torch.equal(aq.q, ref.q)
    assert torch.equal(aq.sf, ref.sf)


@pytest.mark.parametrize("M,H,C", [(4096, 4096, 1024), (300, 384, 256)])
def test_mx_swiglu_dgrad(M, H, C):
    """The MLP backward in MXFP8 (fp8 "mx2"): d(pre) from dy's and W3^T's MX copies with the SwiGLU backward in the
    epilogue, against the bf16 formula on the dequantized operands; its MX copy equals quantizing d(pre) separately."""
    from nano_gpic_b200.ops import gemm as G
    from nano_gpic_b200.ops import mx
    dyq = mx.quant(_input(M, C, 5))
    w3 = (torch.randn(C, H, device="cuda") * 0.05).to(torch.bfloat16)
    w3tq = mx.quant(w3.t().contiguous())
    pre = (torch.randn(M, 2 * H, device="cuda") * 2).to(torch.bfloat16)
    dpre, dq = mx.swiglu_dgrad(dyq, w3tq, pre, quant_out=True)
    ref = G.swiglu_dgrad(dyq.dequant().to(torch.bfloat16).cpu(), w3tq.dequant().t().contiguous().to(torch.bfloat16).cpu(),
                         pre.cpu())
    _close(dpre.cpu(), ref, rtol=2e-2, atol=1e-3)
    assert torch.equal(mx.swiglu_dgrad(dyq, w3tq, pre), dpre)
    sep = mx.quant(dpre)
    assert torch.equal(dq.q, sep.q) and torch.equal(dq.sf, sep.sf)


def test_model_fp8_backward_close_to_bf16():
    """fp8 "mx2" (the MLP dgrads in MXFP8 too): loss-gradient direction stays close to bf16."""
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    torch.manual_seed(0)
    net = JiT_T2I(input_size=64, in_channels=3, num_groups=4, hidden_size=256, num_blocks=2, num_text_blocks=1,
                  patch_size=16, txt_embed_dim=2048, txt_max_length=32).cuda()
    B = 4
    x = torch.randn(B, 3, 64, 64, device="cuda")
    t = torch.rand(B, device="cuda")
    y = torch.randn(B, 32, 2048, device="cuda").to(torch.bfloat16)
    m = torch.ones(B, 32, dtype=torch.bool, device="cuda")
    with torch.no_grad():
        for prm in net.parameters():
            prm.add_(torch.randn_like(prm) * 0.02)
    grads = []
    for mode in (None, "mx2"):
        net.set_fp8(mode)
        net.zero_grad(set_to_none=True)
        o = net(x, t, y, y_mask=m)
        o.float().square().mean().backward()
        grads.append({n: p.grad.clone() for n, p in net.named_parameters() if p.grad is not None})
    for n in ("blocks.0.norm1.weight", "blocks.0.attn.qkv_x.weight", "blocks.1.mlp.w12.weight", "x_embedder.proj2.weight"):
        rel = (grads[1][n] - grads[0][n]).norm() / grads[0][n].norm()
        assert rel < 0.1, (n, rel)
