"""The TF-Inception feature network (nano_gpic_b200/eval/inception.py): the published port's parameter layout, the
pool_3 feature shape, strict loading from a weight file, TF1's bilinear resize (no half-pixel centres) on a hand-worked
case, and fast_eval's inception backend end to end (a weight file of random values stands in for the published one)."""
import json

import numpy as np
import torch

from nano_gpic_b200.eval.inception import FIDInception, resize_tf1_bilinear


def test_layout_and_features():
    m = FIDInception().eval()
    sd = m.state_dict()
    assert len(sd) == 566 and "Mixed_7c.branch3x3dbl_3b.bn.running_var" in sd and sd["fc.weight"].shape == (1008, 2048)
    assert sum(p.numel() for p in m.parameters()) == 23850960
    f = m(torch.randint(0, 256, (2, 40, 40, 3), dtype=torch.uint8))
    assert f.shape == (2, 2048) and torch.isfinite(f).all() and (f >= 0).all()  # after ReLU and average pooling


def test_tf1_resize():
    x = torch.tensor([[[[0.0, 10.0], [20.0, 30.0]]]])
    y = resize_tf1_bilinear(x, 4)  # sources 0, 0.5, 1, 1.5 -> clamped at the last pixel
    want = torch.tensor([[0.0, 5.0, 10.0, 10.0], [10.0, 15.0, 20.0, 20.0], [20.0, 25.0, 30.0, 30.0],
                         [20.0, 25.0, 30.0, 30.0]])
    torch.testing.assert_close(y[0, 0], want)
    z = torch.rand(1, 3, 299, 299)
    assert torch.equal(resize_tf1_bilinear(z, 299), z)


def test_fast_eval_inception_backend(tmp_path):
    from nano_gpic_b200.tools import fast_eval
    torch.manual_seed(0)
    w = tmp_path / "inc.pth"
    torch.save(FIDInception().state_dict(), w)
    rng = np.random.default_rng(0)
    samples = rng.integers(0, 256, (6, 32, 32, 3), dtype=np.uint8)
    np.save(tmp_path / "s.npy", samples)
    ref_feats = rng.random((20, 2048)).astype(np.float32)
    np.savez(tmp_path / "ref.npz", inception_mu=ref_feats.mean(0), inception_sigma=np.cov(ref_feats, rowvar=False),
             inception_embeddings=ref_feats)
    out = tmp_path / "out.json"
    assert fast_eval.main([str(tmp_path / "s.npy"), str(tmp_path / "ref.npz"), str(out), "--backend", "inception",
                           "--inception-weights", str(w), "--batch", "4"]) == 0
    res = json.loads(out.read_text())
    assert res["inception_n"] == 6 and np.isfinite(res["inception_fd"]) and "inception_precision" in res
