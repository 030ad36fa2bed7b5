"""Pillow's 8-bit bicubic resample, bit for bit, with the passes run on the GPU (csrc/resize.cu).

Role of the reference's lever C (baselines/PixelGen/src/data/dataset/pil_exact.py:1-109, pil_exact_gpu.py:1-211;
default on in jobs/train_ladder.sh:138): the data workers decode, box-halve and plan the crop; the two separable
bicubic passes of the random region crop (reference augmentation.py random_crop_arr_region) run on the device for the
whole batch.

Pillow's pass (libImaging/Resample.c) computes each output value as
    clip8((2^21 + sum_x in[xmin + x] * kk[x]) >> 22)                              (int32 sum)
with kk = trunc(w * 2^22 +- 0.5) from double-precision weights w of the a = -0.5 cubic, normalised per output pixel,
and the box edges taken as single-precision floats. `coeffs` restates that arithmetic with IEEE double operations in
the C code's order (sequential weight sums), so the tables, and hence every output byte, equal Pillow's.
The region crop runs each axis as its own Pillow resize call (the order that random_crop_arr_region uses), so the
intermediate is rounded to 8 bits between the passes exactly as there.
"""
import math
import random

import numpy as np

PRECISION_BITS = 22


def cubic(x):
    """Pillow's bicubic filter (a = -0.5) on a float64 array."""
    a = -0.5
    x = np.abs(x)
    near = ((a + 2.0) * x - (a + 3.0)) * x * x + 1
    far = (((x - 5) * x + 8) * x - 4) * a
    return np.where(x < 1.0, near, np.where(x < 2.0, far, 0.0))


def coeffs(in_size, in0, in1, out_size):
    """One pass's tables for input extent in_size, box [in0, in1) and out_size outputs:
    xmin [out] int32 (first input index), xlen [out] int32 (taps used), kk [out, ksize] int32 (fixed-point weights)."""
    f0, f1 = np.float32(in0), np.float32(in1)
    scale = float(np.float32(f1 - f0)) / out_size  # (double)(in1 - in0) / outSize, the difference in float
    fscale = max(scale, 1.0)
    support = 2.0 * fscale
    ksize = int(math.ceil(support)) * 2 + 1
    center = float(f0) + (np.arange(out_size, dtype=np.float64) + 0.5) * scale
    lo = np.maximum(np.trunc(center - support + 0.5), 0).astype(np.int64)
    hi = np.minimum(np.trunc(center + support + 0.5).astype(np.int64), in_size)
    xlen = hi - lo
    taps = np.arange(ksize)[None, :]
    used = taps < xlen[:, None]
    w = np.where(used, cubic(((taps + lo[:, None]).astype(np.float64) - center[:, None] + 0.5) * (1.0 / fscale)), 0.0)
    total = np.cumsum(w, axis=1)[:, -1]  # left-to-right sum (the unused taps add exact zeros)
    safe = np.where(total != 0.0, total, 1.0)
    k = np.where((total != 0.0)[:, None], w / safe[:, None], w)
    s = k * float(1 << PRECISION_BITS)
    kk = np.where(k < 0, np.trunc(-0.5 + s), np.trunc(0.5 + s))
    kk = np.where(used, kk, 0.0)
    return lo.astype(np.int32), xlen.astype(np.int32), kk.astype(np.int32)


def run_pass(arr, axis, xmin, xlen, kk):
    """CPU reference of one pass over an [H, W, C] uint8 array along `axis` (0: rows, 1: columns)."""
    src = np.moveaxis(arr, axis, 0).astype(np.int64)
    n_out, ksize = kk.shape
    acc = np.full((n_out,) + src.shape[1:], 1 << (PRECISION_BITS - 1), dtype=np.int64)
    for j in range(ksize):
        idx = np.minimum(xmin + j, src.shape[0] - 1)  # taps past xlen have weight 0
        acc += src[idx] * kk[:, j].astype(np.int64)[:, None, None]
    return np.moveaxis(np.clip(acc >> PRECISION_BITS, 0, 255).astype(np.uint8), 0, axis)


class CropPlan:
    """A sample's source rows and its two passes [(axis, xmin, xlen, kk), ...] (the first runs on `src`)."""

    __slots__ = ("src", "passes", "box")

    def __init__(self, src, passes, box=None):
        self.src, self.passes, self.box = src, passes, box

    def run_cpu(self):
        out = self.src
        for axis, xmin, xlen, kk in self.passes:
            out = run_pass(out, axis, xmin, xlen, kk)
        return out


def plan_random_crop(pil_image, image_size, min_crop_frac=0.8, max_crop_frac=1.0, rng=random):
    """random_crop_arr_region's draws and box halvings (in Pillow), returned as a CropPlan of its two resize calls:
    the short side goes to a random size in [size / max_frac, size / min_frac], then a random size x size window of
    that resized image is produced by resizing only the window's box. Running the plan equals the reference's crop
    bit for bit."""
    from PIL import Image
    smallest = rng.randrange(math.ceil(image_size / max_crop_frac), math.ceil(image_size / min_crop_frac) + 1)
    img = pil_image
    while min(*img.size) >= 2 * smallest:
        img = img.resize(tuple(x // 2 for x in img.size), resample=Image.BOX)
    W, H = img.size
    s = smallest / min(W, H)
    ow, oh = round(W * s), round(H * s)
    cy = rng.randrange(oh - image_size + 1)
    cx = rng.randrange(ow - image_size + 1)
    sx, sy = W / ow, H / oh
    x0, x1 = cx * sx, min(W, (cx + image_size) * sx)
    y0, y1 = cy * sy, min(H, (cy + image_size) * sy)
    arr = np.asarray(img, dtype=np.uint8)
    if (H - oh) > 0 and (H - oh) > (W - ow) * 2:
        # rows first over the whole width (Pillow's order for this shape), then columns
        return CropPlan(arr, [(0,) + coeffs(H, y0, y1, image_size), (1,) + coeffs(W, x0, x1, image_size)],
                        (0, H, x0, x1, y0, y1, True))
    # columns first, on the source rows the row pass can reach (bicubic support 2 x the row scale)
    sup = 2 * max(1.0, sy)
    r0, r1 = max(0, int(y0 - sup) - 1), min(H, int(y1 + sup) + 2)
    return CropPlan(np.ascontiguousarray(arr[r0:r1]),
                    [(1,) + coeffs(W, x0, x1, image_size), (0,) + coeffs(r1 - r0, y0 - r0, y1 - r0, image_size)],
                    (r0, r1, x0, x1, y0, y1, False))


def pillow_region_crop(pil_image, plan_args, image_size):
    """The same crop through Pillow's own resize calls (the oracle of the tests): plan_args = a plan's box
    (r0, r1, x0, x1, y0, y1, rows_first), pil_image = the box-halved image the plan was made from."""
    from PIL import Image
    r0, r1, x0, x1, y0, y1, rows_first = plan_args
    W, H = pil_image.size
    if rows_first:
        tmp = pil_image.resize((W, image_size), resample=Image.BICUBIC, box=(0, y0, W, y1))
        return np.asarray(tmp.resize((image_size, image_size), resample=Image.BICUBIC, box=(x0, 0, x1, image_size)))
    tmp = pil_image.crop((0, r0, W, r1)).resize((image_size, r1 - r0), resample=Image.BICUBIC,
                                                box=(x0, 0, x1, r1 - r0))
    return np.asarray(tmp.resize((image_size, image_size), resample=Image.BICUBIC,
                                 box=(0, y0 - r0, image_size, y1 - r0)))


# ------------------------------------------------------------------------------------------------ batch on the GPU
class ResizeBatch:
    """A batch of CropPlans packed for csrc/resize.cu: sources (uint8), tables (int32) and per-sample descriptors.
    `run(device)` returns the crops as a [B, size, size, 3] uint8 device tensor."""

    def __init__(self, plans, image_size, pin=False):
        import torch
        self.size = image_size
        B = len(plans)
        srcs, tabs = [], []
        desc = np.zeros((B, 16), dtype=np.int64)
        s_pos = t_pos = m_pos = 0
        for i, p in enumerate(plans):
            h, w = p.src.shape[:2]
            (a0, xm0, xl0, k0), (a1, xm1, xl1, k1) = p.passes
            mid = (h, image_size) if a0 == 1 else (image_size, w)  # shape after the first pass
            t0 = np.concatenate([xm0, xl0, k0.ravel()])
            t1 = np.concatenate([xm1, xl1, k1.ravel()])
            desc[i] = [s_pos, h, w, a0, k0.shape[1], t_pos, m_pos, mid[0], mid[1], a1, k1.shape[1],
                       t_pos + t0.size, 0, 0, 0, 0]
            srcs.append(p.src.reshape(-1))
            tabs += [t0, t1]
            s_pos += p.src.size + (-p.src.size) % 16
            if (-p.src.size) % 16:
                srcs.append(np.zeros((-p.src.size) % 16, dtype=np.uint8))
            t_pos += t0.size + t1.size
            m_pos += mid[0] * mid[1] * 3
        self.src = torch.from_numpy(np.concatenate(srcs))
        self.tab = torch.from_numpy(np.concatenate(tabs).astype(np.int32))
        self.desc = torch.from_numpy(desc)
        self.tmp_bytes = m_pos
        if pin:
            self.src, self.tab, self.desc = self.src.pin_memory(), self.tab.pin_memory(), self.desc.pin_memory()

    def __len__(self):
        return self.desc.shape[0]

    def pin_memory(self):
        """Called by the DataLoader's pinning thread: page-locked buffers for the asynchronous copies of run()."""
        self.src, self.tab, self.desc = self.src.pin_memory(), self.tab.pin_memory(), self.desc.pin_memory()
        return self

    def run(self, device):
        import torch
        from .._ext import ext
        src = self.src.to(device, non_blocking=True)
        tab = self.tab.to(device, non_blocking=True)
        desc = self.desc.to(device, non_blocking=True)
        tmp = torch.empty(self.tmp_bytes, dtype=torch.uint8, device=device)
        out = torch.empty(len(self), self.size, self.size, 3, dtype=torch.uint8, device=device)
        ext().resize_passes(src, tab, desc, tmp, out, int(self.desc[:, 1].max()), int(self.desc[:, 2].max()))
        return out

    def run_cpu(self, plans):
        return np.stack([p.run_cpu() for p in plans])
