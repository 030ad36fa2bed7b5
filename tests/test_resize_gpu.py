"""The batched bicubic crop passes on the GPU (csrc/resize.cu) equal the CPU plans (and hence Pillow) byte for byte."""
import random

import numpy as np
import pytest
import torch
from PIL import Image

from nano_gpic_b200.data import pil_resize as PR

pytestmark = pytest.mark.gpu


def test_gpu_batch_equals_cpu():
    rng = np.random.default_rng(0)
    shapes = [(300, 400), (1000, 257), (2000, 1500), (257, 1000), (640, 480), (321, 321)] * 3
    plans = []
    for i, (h, w) in enumerate(shapes):
        img = Image.fromarray(rng.integers(0, 256, (h, w, 3), dtype=np.uint8))
        plans.append(PR.plan_random_crop(img, 256, rng=random.Random(i)))
    batch = PR.ResizeBatch(plans, 256).pin_memory()
    got = batch.run(torch.device("cuda")).cpu().numpy()
    ref = np.stack([p.run_cpu() for p in plans])
    assert got.shape == (len(plans), 256, 256, 3)
    assert np.array_equal(got, ref), int((got != ref).sum())
