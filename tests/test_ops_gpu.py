"""CUDA kernels of the norm, q/k-prep and attention ops against the same ops' fp32 PyTorch paths (run on CPU copies)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(a, b, rtol=2e-2, atol=2e-2, what=""):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= atol + rtol * ref, f"{what}: max err {err} vs ref max {ref}"


def _cpu(*ts):
    return [t.cpu() if isinstance(t, torch.Tensor) else t for t in ts]


@pytest.mark.parametrize("mod", [True, False])
@pytest.mark.parametrize("M,C,rpg", [(512, 1024, 256), (520, 768, 40), (96, 64, 96)])
def test_rms_mod(mod, M, C, rpg):
    from nano_gpic_b200.ops import norm
    G = (M + rpg - 1) // rpg
    x = torch.randn(M, C, device="cuda").bfloat16()
    w = torch.rand(C, device="cuda") + 0.5
    m = (torch.randn(G, 6 * C, device="cuda") * 0.3).bfloat16()
    sh, sc = (m[:, :C], m[:, C:2 * C]) if mod else (None, None)
    h, r = norm.rms_mod_fwd(x, w, sh, sc, rpg)
    hc, rc = norm.rms_mod_fwd(*_cpu(x, w, sh, sc), rpg)
    _close(h, hc, what="h")
    _close(r, rc, rtol=1e-3, atol=1e-3, what="rstd")
    dh = torch.randn(M, C, device="cuda").bfloat16()
    dres = torch.randn(M, C, device="cuda").bfloat16()
    dw = torch.zeros(C, device="cuda")
    dmod = torch.zeros(G, 6 * C, device="cuda")
    dx = norm.rms_mod_bwd(dh, x, r, w, sc, rpg, dres=dres, dw_acc=dw,
                          dshift=dmod[:, :C] if mod else None, dscale=dmod[:, C:2 * C] if mod else None)
    dwc = torch.zeros(C)
    dmodc = torch.zeros(G, 6 * C)
    dxc = norm.rms_mod_bwd(*_cpu(dh, x, rc, w, sc), rpg, dres=dres.cpu(), dw_acc=dwc,
                           dshift=dmodc[:, :C] if mod else None, dscale=dmodc[:, C:2 * C] if mod else None)
    _close(dx, dxc, what="dx")
    _close(dw, dwc, rtol=1e-2, atol=1e-2, what="dw")
    _close(dmod, dmodc, rtol=1e-2, atol=1e-2, what="dmod")


def test_layernorm():
    from nano_gpic_b200.ops import norm
    x = (torch.randn(700, 1024, device="cuda") * 3 + 1).bfloat16()
    h, mu, r = norm.layernorm_fwd(x)
    hc, muc, rc = norm.layernorm_fwd(x.cpu())
    _close(h, hc, what="h")
    dh = torch.randn_like(x)
    _close(norm.layernorm_bwd(dh, x, mu, r), norm.layernorm_bwd(dh.cpu(), x.cpu(), muc, rc), what="dx")


@pytest.mark.parametrize("rope", [True, False])
def test_qk_norm(rope):
    from nano_gpic_b200.ops import qk
    from nano_gpic_b200.models.layers import rope_tables
    B, L, H = 3, 256, 4
    qkv = torch.randn(B * L, 3 * H * 64, device="cuda").bfloat16()
    src = qkv[:, H * 64:2 * H * 64]
    w = torch.rand(64, device="cuda") + 0.5
    cos, sin = rope_tables(64, 16, 16, device="cuda") if rope else (None, None)
    out, r = qk.qk_norm_fwd(src, w, cos, sin, L)
    outc, rc = qk.qk_norm_fwd(*_cpu(src, w, cos, sin), L)
    _close(out, outc, what="out")
    d = torch.randn_like(out)
    dsrc = torch.zeros_like(qkv)
    dw = torch.zeros(64, device="cuda")
    qk.qk_norm_bwd(d, src, r, w, cos, sin, L, dsrc=dsrc[:, H * 64:2 * H * 64], dw_acc=dw)
    dwc = torch.zeros(64)
    dxc = qk.qk_norm_bwd(*_cpu(d, src, rc, w, cos, sin), L, dw_acc=dwc)
    _close(dsrc[:, H * 64:2 * H * 64], dxc, what="dx")
    assert dsrc[:, :H * 64].abs().max() == 0
    _close(dw, dwc, rtol=1e-2, atol=1e-2, what="dw")


@pytest.mark.parametrize("joint", [True, False])
def test_attention(joint):
    from nano_gpic_b200.ops import attention as A
    torch.manual_seed(0)
    B, H = 3, 2
    C = H * 64
    if joint:
        Lq, L0, L1 = 256, 256, 72
        n0 = 256
        n1 = torch.tensor([72, 5, 40], dtype=torch.int32, device="cuda")
    else:
        Lq, L0, L1 = 72, 72, 0
        n0 = torch.tensor([72, 9, 33], dtype=torch.int32, device="cuda")
        n1 = None
    qkv = torch.randn(B * Lq, 3 * C, device="cuda").bfloat16()
    q, k0, v0 = qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:]
    if joint:
        kv = torch.randn(B * L1, 2 * C, device="cuda").bfloat16()
        k1, v1 = kv[:, :C], kv[:, C:]
    else:
        k1 = v1 = None
    o, lse = A.attn_fwd(q, Lq, k0, v0, L0, n0, k1, v1, L1, n1)
    oc, lsec = A.attn_fwd(*_cpu(q), Lq, *_cpu(k0, v0), L0, n0 if isinstance(n0, int) else n0.cpu(),
                          *_cpu(k1, v1), L1, n1.cpu() if n1 is not None else None)
    _close(o, oc, what="o")
    _close(lse, lsec, rtol=1e-3, atol=1e-3, what="lse")
    do = torch.randn_like(o)
    g = A.attn_bwd(do, q, Lq, k0, v0, L0, n0, o, lse, k1, v1, L1, n1)
    gc = A.attn_bwd(*_cpu(do, q), Lq, *_cpu(k0, v0), L0, n0 if isinstance(n0, int) else n0.cpu(), *_cpu(oc, lsec, k1, v1),
                    L1, n1.cpu() if n1 is not None else None)
    for name, a, b in zip(["dq", "dk0", "dv0", "dk1", "dv1"], g, gc):
        if a is None:
            continue
        _close(a, b, what=name)


@pytest.mark.parametrize("case", ["joint", "text", "joint_long", "text_long", "odd"])
def test_attention_tc_forward(case):
    """tcgen05 forward against the fp32 reference and the mma.sync kernel (partial tiles, skipped tiles, T > 128)."""
    from nano_gpic_b200.ops import attention as A
    torch.manual_seed(1)
    B, H = 3, 4
    C = H * 64
    if case == "joint":
        Lq, L0, L1, n0, n1 = 256, 256, 72, 256, torch.tensor([72, 5, 40], dtype=torch.int32, device="cuda")
    elif case == "joint_long":
        Lq, L0, L1, n0, n1 = 256, 256, 200, 256, torch.tensor([200, 129, 3], dtype=torch.int32, device="cuda")
    elif case == "text_long":  # several query-tile pairs per sample, tile B of the last pair past the queries
        Lq, L0, L1, n0, n1 = 320, 320, 0, torch.tensor([320, 130, 1], dtype=torch.int32, device="cuda"), None
    elif case == "odd":
        Lq, L0, L1, n0, n1 = 200, 200, 40, torch.tensor([200, 150, 7], dtype=torch.int32, device="cuda"), \
            torch.tensor([40, 0, 17], dtype=torch.int32, device="cuda")
    else:
        Lq, L0, L1, n0, n1 = 72, 72, 0, torch.tensor([72, 9, 33], dtype=torch.int32, device="cuda"), None
    qkv = torch.randn(B * Lq, 3 * C, device="cuda").bfloat16()
    q, k0, v0 = qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:]
    if L1:
        kv = torch.randn(B * L1, 2 * C, device="cuda").bfloat16()
        k1, v1 = kv[:, :C], kv[:, C:]
    else:
        k1 = v1 = None
    o, lse = A.attn_fwd(q, Lq, k0, v0, L0, n0, k1, v1, L1, n1, impl="tc")
    o1, lse1 = A.attn_fwd(q, Lq, k0, v0, L0, n0, k1, v1, L1, n1, impl="tc1")
    _close(o, o1, rtol=1e-2, atol=1e-2, what="o: version 3 vs one-tile kernel")
    o2, lse2 = A.attn_fwd(q, Lq, k0, v0, L0, n0, k1, v1, L1, n1, impl="tc2")
    _close(o, o2, rtol=1e-2, atol=1e-2, what="o: version 3 vs version 2")
    _close(lse, lse2, rtol=1e-4, atol=1e-4, what="lse: version 3 vs version 2")
    om, lsem = A.attn_fwd(q, Lq, k0, v0, L0, n0, k1, v1, L1, n1, impl="mma")
    oc, lsec = A.attn_fwd(*_cpu(q), Lq, *_cpu(k0, v0), L0, n0 if isinstance(n0, int) else n0.cpu(),
                          *_cpu(k1, v1), L1, n1.cpu() if n1 is not None else None)
    _close(o, oc, what="o vs fp32")
    _close(lse, lsec, rtol=1e-3, atol=2e-3, what="lse vs fp32")
    _close(o, om, what="o vs mma")
    from nano_gpic_b200.ops import status
    assert status.read() == 0


@pytest.mark.parametrize("case", ["joint", "text", "joint_long", "odd", "text_long"])
def test_attention_tc_backward(case):
    """tcgen05 backward against the fp32 autograd reference and the mma.sync kernels; dK/dV of padded keys are zero."""
    from nano_gpic_b200.ops import attention as A
    torch.manual_seed(2)
    B, H = 3, 4
    C = H * 64
    if case == "joint":
        Lq, L0, L1, n0, n1 = 256, 256, 72, 256, torch.tensor([72, 5, 40], dtype=torch.int32, device="cuda")
    elif case == "joint_long":
        Lq, L0, L1, n0, n1 = 256, 256, 200, 256, torch.tensor([200, 129, 3], dtype=torch.int32, device="cuda")
    elif case == "odd":
        Lq, L0, L1, n0, n1 = 200, 200, 40, torch.tensor([200, 150, 7], dtype=torch.int32, device="cuda"), \
            torch.tensor([40, 0, 17], dtype=torch.int32, device="cuda")
    elif case == "text_long":  # 3 key tiles, the third one dead for two samples
        Lq, L0, L1, n0, n1 = 320, 320, 0, torch.tensor([320, 130, 1], dtype=torch.int32, device="cuda"), None
    else:
        Lq, L0, L1, n0, n1 = 72, 72, 0, torch.tensor([72, 9, 33], dtype=torch.int32, device="cuda"), None
    qkv = torch.randn(B * Lq, 3 * C, device="cuda").bfloat16()
    q, k0, v0 = qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:]
    if L1:
        kv = torch.randn(B * L1, 2 * C, device="cuda").bfloat16()
        k1, v1 = kv[:, :C], kv[:, C:]
    else:
        k1 = v1 = None
    o, lse = A.attn_fwd(q, Lq, k0, v0, L0, n0, k1, v1, L1, n1)
    do = torch.randn_like(o)
    g1 = A.attn_bwd(do, q, Lq, k0, v0, L0, n0, o, lse, k1, v1, L1, n1, impl="tc1")
    g2 = A.attn_bwd(do, q, Lq, k0, v0, L0, n0, o, lse, k1, v1, L1, n1, impl="tc2")
    dqkv = torch.full_like(qkv, 7.0)  # strided destinations, like the fused qkv gradient
    dkv = torch.full((B * L1, 2 * C), 7.0, device="cuda", dtype=torch.bfloat16) if L1 else None
    g = A.attn_bwd(do, q, Lq, k0, v0, L0, n0, o, lse, k1, v1, L1, n1, dq=dqkv[:, :C], dk0=dqkv[:, C:2 * C],
                   dv0=dqkv[:, 2 * C:], dk1=dkv[:, :C] if L1 else None, dv1=dkv[:, C:] if L1 else None, impl="tc")
    gm = A.attn_bwd(do, q, Lq, k0, v0, L0, n0, o, lse, k1, v1, L1, n1, impl="mma")
    n0c = n0 if isinstance(n0, int) else n0.cpu()
    gc = A.attn_bwd(*_cpu(do, q), Lq, *_cpu(k0, v0), L0, n0c, *_cpu(o, lse, k1, v1), L1,
                    n1.cpu() if n1 is not None else None)
    for name, a, m, c, a1, a2 in zip(["dq", "dk0", "dv0", "dk1", "dv1"], g, gm, gc, g1, g2):
        if a is None:
            continue
        _close(a, c, what=name + " vs fp32")
        _close(a, m, what=name + " vs mma")
        _close(a, a1, rtol=1e-2, atol=1e-2, what=name + " version 3 vs one CTA per key tile")
        _close(a, a2, rtol=1e-2, atol=1e-2, what=name + " version 3 vs version 2")
    from nano_gpic_b200.ops import status
    assert status.read() == 0


def test_u8_to_unit_matches_torch_formula():
    """uint8 HWC -> fp32 CHW in [-1, 1] in one kernel pass, bit-identical to ToTensor + Normalize(0.5, 0.5)."""
    from nano_gpic_b200.train.trainer import uint8_to_float
    img = torch.randint(0, 256, (3, 40, 64, 3), dtype=torch.uint8, device="cuda")
    ref = (((img.permute(0, 3, 1, 2).float() / 255.0) - 0.5) / 0.5).contiguous()
    got = uint8_to_float(img)
    assert got.shape == ref.shape
    if not torch.equal(got, ref):  # at most one rounding step apart where PyTorch rounds differently
        assert (got - ref).abs().max().item() <= 2.0 ** -23, (got - ref).abs().max().item()
