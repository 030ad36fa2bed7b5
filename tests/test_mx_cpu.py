"""MXFP8 quantization rule and scale-factor layout (the PyTorch restatement that the CUDA quantizer is tested against),
and the model's MXFP8 forward on the CPU paths."""
import torch

from nano_gpic_b200.ops import mx


def test_scale_rule_and_layout():
    R, K = 200, 256
    torch.manual_seed(0)
    x = (torch.randn(R, K) * 3).to(torch.bfloat16)
    x[3, :32] = 0
    q = mx.quant(x)
    assert q.q.shape == (R, K) and q.sf.shape == (mx.rows_pad(R) // 128, K // 128, 512)
    e = q.scales()
    amax = x.float().view(R, K // 32, 32).abs().amax(-1)
    # the smallest power of two with amax / 2^e <= 448
    nz = amax > 0
    assert (amax[nz] / torch.pow(2.0, e[nz].float()) <= 448).all()
    assert (amax[nz] / torch.pow(2.0, e[nz].float() - 1) > 448).all()
    assert e[3, 0] == 0
    # the byte of row r, k-block j sits at block (r // 128, j // 4), offset (r % 32) * 16 + (r // 32 % 4) * 4 + j % 4
    r, j = 137, 5
    byte = q.sf[r // 128, j // 4, (r % 32) * 16 + (r // 32 % 4) * 4 + j % 4]
    assert int(byte) - 127 == int(e[r, j])
    # padding rows hold scale 1
    pad = q.sf.view(-1, K // 128, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(-1, K // 32)[R:]
    assert (pad == 127).all()


def test_dequant_error_bound():
    R, K = 64, 128
    x = torch.randn(R, K).to(torch.bfloat16)
    d = mx.quant(x).dequant()
    blk = x.float().view(R, K // 32, 32).abs().amax(-1, keepdim=True)
    assert ((d - x.float()).view(R, K // 32, 32).abs() <= blk * 2.0 ** -4).all()


def test_model_fp8_cpu_runs_and_is_close():
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    torch.manual_seed(0)
    net = JiT_T2I(input_size=32, in_channels=3, num_groups=2, hidden_size=128, num_blocks=1, num_text_blocks=1,
                  patch_size=16, txt_embed_dim=2048, txt_max_length=8)
    x = torch.randn(2, 3, 32, 32)
    t = torch.rand(2)
    y = torch.randn(2, 8, 2048).to(torch.bfloat16)
    m = torch.ones(2, 8, dtype=torch.bool)
    with torch.no_grad():  # the zero-initialised output and gate layers would make every output 0
        for prm in net.parameters():
            prm.add_(torch.randn_like(prm) * 0.02)
    outs = []
    grads = []
    for mode in (None, "mx", "mx2"):
        net.set_fp8(mode)
        net.zero_grad(set_to_none=True)
        o = net(x, t, y, y_mask=m)
        o.float().square().mean().backward()
        outs.append(o.float().detach())
        grads.append(net.blocks[0].mlp.w12.weight.grad.clone())
    assert net.blocks[0].mlp.w3.weight.grad is not None
    assert (outs[1] - outs[0]).norm() / outs[0].norm() < 0.05
    assert torch.equal(outs[2], outs[1])  # mx2 changes the backward only
    assert (grads[2] - grads[0]).norm() / grads[0].norm() < 0.1
