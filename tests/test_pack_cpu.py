"""Packed captions (the reference's lever E, y_pack; JiT_T2I.py:54-65 there) on the CPU paths: the same model run on
the padded captions with a mask and on the packed rows gives the same prediction and the same gradient for every
parameter (the reference states the packed path is the masked path's math); pack_captions builds the reference's
y_pack fields."""
import torch

TINY = dict(input_size=64, in_channels=3, num_groups=2, hidden_size=128, num_blocks=2, num_text_blocks=2,
            patch_size=16, txt_embed_dim=32, txt_max_length=24, bottleneck_dim=16)


def _model(seed=0):
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    torch.manual_seed(seed)
    m = JiT_T2I(**TINY)
    with torch.no_grad():  # non-zero adaLN / final layer, so every path carries signal
        for p in m.parameters():
            if p.requires_grad:
                p.copy_(torch.randn_like(p) * (0.2 if p.ndim == 2 else 0.05) + (1.0 if p.ndim == 1 and p.numel() in
                                                                                   (64, 128) else 0.0))
    return m


def _inputs(lens, T, seed=1):
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    x = torch.rand(B, 3, 64, 64, generator=g) * 2 - 1
    t = torch.rand(B, generator=g)
    y = torch.randn(B, T, 32, generator=g)
    mask = torch.arange(T)[None] < torch.tensor(lens)[:, None]
    y = y * mask[..., None]
    return x, t, y, mask


def test_pack_captions_fields():
    from nano_gpic_b200.parallel.rebalance import pack_captions
    _, _, y, mask = _inputs([3, 7, 1], 8)
    yp, pk = pack_captions(y, mask, bucket=16)
    assert yp.shape == (16, 32)
    assert pk["cu"].tolist() == [0, 3, 10, 11] and pk["lens"].tolist() == [3, 7, 1]
    assert pk["pidx"][:11].tolist() == [0, 1, 2, 8, 9, 10, 11, 12, 13, 14, 16] and set(pk["pidx"][11:].tolist()) == {24}
    assert pk["pos"][:11].tolist() == [0, 1, 2, 0, 1, 2, 3, 4, 5, 6, 0] and pk["real"].sum() == 11
    assert torch.equal(pk["onehot"].sum(1)[:11], torch.ones(11, dtype=torch.long)) and not pk["onehot"][11:].any()
    assert torch.equal(yp[3:10], y[1, :7]) and not yp[11:].any()


def test_packed_matches_masked():
    from nano_gpic_b200.parallel.rebalance import pack_captions
    lens, T = [5, 12, 1], 12
    x, t, y, mask = _inputs(lens, T)
    w = torch.randn(3, 3, 64, 64, generator=torch.Generator().manual_seed(3))
    grads, outs = [], []
    for packed in (False, True):
        m = _model()
        if packed:
            yp, pk = pack_captions(y, mask, bucket=8)  # 18 real rows + 6 dummy rows
            out = m(x, t, yp, y_pack=pk)
        else:
            out = m(x, t, y, y_mask=mask)
        (out.float() * w).sum().backward()
        outs.append(out.float().detach())
        grads.append({n: p.grad.clone() for n, p in m.named_parameters() if p.requires_grad})
    torch.testing.assert_close(outs[1], outs[0], rtol=1e-3, atol=1e-3)
    bad = []
    for n, g0 in grads[0].items():
        g1 = grads[1][n]
        e = (g1 - g0).norm().item() / (g0.norm().item() + 1e-8)
        if e > 1e-4:
            bad.append((n, round(e, 4)))
    assert not bad, bad
