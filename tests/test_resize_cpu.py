"""Pillow-exact bicubic crop plans (data/pil_resize.py) against Pillow's own resize calls, byte for byte."""
import random

import numpy as np
import pytest
from PIL import Image

from nano_gpic_b200.data import pil_resize as PR

SHAPES = [(300, 400), (400, 300), (257, 1000), (1000, 257), (640, 480), (2000, 1500), (321, 321), (256, 900)]


def _image(h, w, seed, smooth):
    rng = np.random.default_rng(seed)
    if smooth:
        y, x = np.mgrid[0:h, 0:w]
        a = np.stack([(x * 255 // max(w - 1, 1)), (y * 255 // max(h - 1, 1)), ((x + y) * 7) % 256], -1)
        return Image.fromarray(a.astype(np.uint8))
    return Image.fromarray(rng.integers(0, 256, (h, w, 3), dtype=np.uint8))


def _halved(img, size, seed):
    """The image the plan resizes (the same draw of the short side and the same BOX halvings)."""
    import math
    rng = random.Random(seed)
    smallest = rng.randrange(math.ceil(size / 1.0), math.ceil(size / 0.8) + 1)
    while min(*img.size) >= 2 * smallest:
        img = img.resize(tuple(x // 2 for x in img.size), resample=Image.BOX)
    return img


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("smooth", [False, True])
def test_plan_equals_pillow(shape, smooth):
    size = 256
    for seed in range(4):
        img = _image(*shape, seed, smooth)
        plan = PR.plan_random_crop(img, size, rng=random.Random(seed))
        got = plan.run_cpu()
        ref = PR.pillow_region_crop(_halved(img, size, seed), plan.box, size)
        assert got.shape == (size, size, 3)
        assert np.array_equal(got, ref), (shape, seed, int((got != ref).sum()))


def test_coeffs_match_pillow_single_pass():
    """One horizontal pass with a fractional box: the tables reproduce Pillow's output row."""
    img = _image(5, 777, 3, smooth=False)
    for box in [(0.0, 777.0), (13.37, 600.25), (101.5, 357.75)]:
        ref = np.asarray(img.resize((256, 5), resample=Image.BICUBIC, box=(box[0], 0, box[1], 5)))
        xmin, xlen, kk = PR.coeffs(777, box[0], box[1], 256)
        got = PR.run_pass(np.asarray(img), 1, xmin, xlen, kk)
        assert np.array_equal(got, ref), box


def test_batch_packing_layout():
    plans = [PR.plan_random_crop(_image(*s, i, False), 256, rng=random.Random(i)) for i, s in enumerate(SHAPES[:4])]
    b = PR.ResizeBatch(plans, 256)
    assert len(b) == 4
    d = b.desc.numpy()
    for i, p in enumerate(plans):
        h, w = p.src.shape[:2]
        assert (d[i, 1], d[i, 2]) == (h, w)
        assert d[i, 0] % 16 == 0
        src = b.src.numpy()[d[i, 0]:d[i, 0] + h * w * 3].reshape(h, w, 3)
        assert np.array_equal(src, p.src)
        a0, xm0, xl0, k0 = p.passes[0]
        t = b.tab.numpy()[d[i, 5]:d[i, 5] + 2 * 256 + k0.size]
        assert np.array_equal(t[:256], xm0) and np.array_equal(t[256:512], xl0)
        assert np.array_equal(t[512:], k0.ravel())
