"""Inception-v3 pool features for FID-style metrics: the role of the reference's TF-Inception backend
(gpic_eval/backends/inception.py:139, tools/official_inception_sharded.py:1-55), which runs TensorFlow's
`classify_image_graph_def.pb` and reads its 2048-d `pool_3` output.

This is the same network written as a PyTorch module, in the layout of the published PyTorch port of that graph's
weights (`pt_inception-2015-12-05-*.pth`, the FID Inception weights): conv + batch norm (eps 1e-3) + ReLU units, the
Inception A-E blocks of Szegedy et al. 2016 ("Rethinking the Inception Architecture"), with the TF graph's own
choices where they differ from the torchvision classifier: average pools that do not count padding in blocks A, C
and the first E block, a max pool in the last E block's pool branch, and 1008 logits. The input path follows the TF
graph too: float pixels 0..255, bilinear resize to 299 x 299 WITHOUT half-pixel centres (TF1's ResizeBilinear:
source = destination * in / out), then (x - 128) / 128.

The weights are not in this repository and cannot be fetched on a machine without network access: pass the file
(`FIDInception.from_file(path)` or GPIC_INCEPTION_WEIGHTS). Without it the module still runs (random weights) for
tests of the plumbing; its features are then not comparable with published numbers.
"""
import os

import torch
import torch.nn as nn
import torch.nn.functional as F


class Unit(nn.Module):
    """conv (no bias) -> batch norm (eps 1e-3) -> ReLU; `conv` / `bn` keep the port's parameter names."""

    def __init__(self, cin, cout, kernel, stride=1, padding=0):
        super().__init__()
        self.conv = nn.Conv2d(cin, cout, kernel, stride=stride, padding=padding, bias=False)
        self.bn = nn.BatchNorm2d(cout, eps=0.001)

    def forward(self, x):
        return F.relu(self.bn(self.conv(x)))


def _avg3(x):
    return F.avg_pool2d(x, 3, stride=1, padding=1, count_include_pad=False)


class BlockA(nn.Module):
    """35 x 35: 1x1 | 1x1 -> 5x5 | 1x1 -> 3x3 -> 3x3 | avg pool -> 1x1."""

    def __init__(self, cin, pool_ch):
        super().__init__()
        self.branch1x1 = Unit(cin, 64, 1)
        self.branch5x5_1 = Unit(cin, 48, 1)
        self.branch5x5_2 = Unit(48, 64, 5, padding=2)
        self.branch3x3dbl_1 = Unit(cin, 64, 1)
        self.branch3x3dbl_2 = Unit(64, 96, 3, padding=1)
        self.branch3x3dbl_3 = Unit(96, 96, 3, padding=1)
        self.branch_pool = Unit(cin, pool_ch, 1)

    def forward(self, x):
        b5 = self.branch5x5_2(self.branch5x5_1(x))
        b3 = self.branch3x3dbl_3(self.branch3x3dbl_2(self.branch3x3dbl_1(x)))
        return torch.cat([self.branch1x1(x), b5, b3, self.branch_pool(_avg3(x))], 1)


class BlockB(nn.Module):
    """35 -> 17 reduction: 3x3 stride 2 | 1x1 -> 3x3 -> 3x3 stride 2 | max pool."""

    def __init__(self, cin):
        super().__init__()
        self.branch3x3 = Unit(cin, 384, 3, stride=2)
        self.branch3x3dbl_1 = Unit(cin, 64, 1)
        self.branch3x3dbl_2 = Unit(64, 96, 3, padding=1)
        self.branch3x3dbl_3 = Unit(96, 96, 3, stride=2)

    def forward(self, x):
        b3 = self.branch3x3dbl_3(self.branch3x3dbl_2(self.branch3x3dbl_1(x)))
        return torch.cat([self.branch3x3(x), b3, F.max_pool2d(x, 3, stride=2)], 1)


class BlockC(nn.Module):
    """17 x 17 with factorised 7x7 convolutions (1x7 and 7x1)."""

    def __init__(self, cin, c7):
        super().__init__()
        self.branch1x1 = Unit(cin, 192, 1)
        self.branch7x7_1 = Unit(cin, c7, 1)
        self.branch7x7_2 = Unit(c7, c7, (1, 7), padding=(0, 3))
        self.branch7x7_3 = Unit(c7, 192, (7, 1), padding=(3, 0))
        self.branch7x7dbl_1 = Unit(cin, c7, 1)
        self.branch7x7dbl_2 = Unit(c7, c7, (7, 1), padding=(3, 0))
        self.branch7x7dbl_3 = Unit(c7, c7, (1, 7), padding=(0, 3))
        self.branch7x7dbl_4 = Unit(c7, c7, (7, 1), padding=(3, 0))
        self.branch7x7dbl_5 = Unit(c7, 192, (1, 7), padding=(0, 3))
        self.branch_pool = Unit(cin, 192, 1)

    def forward(self, x):
        b7 = self.branch7x7_3(self.branch7x7_2(self.branch7x7_1(x)))
        d = x
        for u in (self.branch7x7dbl_1, self.branch7x7dbl_2, self.branch7x7dbl_3, self.branch7x7dbl_4,
                  self.branch7x7dbl_5):
            d = u(d)
        return torch.cat([self.branch1x1(x), b7, d, self.branch_pool(_avg3(x))], 1)


class BlockD(nn.Module):
    """17 -> 8 reduction: 1x1 -> 3x3 stride 2 | 1x1 -> 1x7 -> 7x1 -> 3x3 stride 2 | max pool."""

    def __init__(self, cin):
        super().__init__()
        self.branch3x3_1 = Unit(cin, 192, 1)
        self.branch3x3_2 = Unit(192, 320, 3, stride=2)
        self.branch7x7x3_1 = Unit(cin, 192, 1)
        self.branch7x7x3_2 = Unit(192, 192, (1, 7), padding=(0, 3))
        self.branch7x7x3_3 = Unit(192, 192, (7, 1), padding=(3, 0))
        self.branch7x7x3_4 = Unit(192, 192, 3, stride=2)

    def forward(self, x):
        b3 = self.branch3x3_2(self.branch3x3_1(x))
        b7 = self.branch7x7x3_4(self.branch7x7x3_3(self.branch7x7x3_2(self.branch7x7x3_1(x))))
        return torch.cat([b3, b7, F.max_pool2d(x, 3, stride=2)], 1)


class BlockE(nn.Module):
    """8 x 8 with split 1x3 / 3x1 outputs; `max_pool` selects the pool branch of the graph's last block."""

    def __init__(self, cin, max_pool=False):
        super().__init__()
        self.max_pool = max_pool
        self.branch1x1 = Unit(cin, 320, 1)
        self.branch3x3_1 = Unit(cin, 384, 1)
        self.branch3x3_2a = Unit(384, 384, (1, 3), padding=(0, 1))
        self.branch3x3_2b = Unit(384, 384, (3, 1), padding=(1, 0))
        self.branch3x3dbl_1 = Unit(cin, 448, 1)
        self.branch3x3dbl_2 = Unit(448, 384, 3, padding=1)
        self.branch3x3dbl_3a = Unit(384, 384, (1, 3), padding=(0, 1))
        self.branch3x3dbl_3b = Unit(384, 384, (3, 1), padding=(1, 0))
        self.branch_pool = Unit(cin, 192, 1)

    def forward(self, x):
        s = self.branch3x3_1(x)
        b3 = torch.cat([self.branch3x3_2a(s), self.branch3x3_2b(s)], 1)
        d = self.branch3x3dbl_2(self.branch3x3dbl_1(x))
        bd = torch.cat([self.branch3x3dbl_3a(d), self.branch3x3dbl_3b(d)], 1)
        p = F.max_pool2d(x, 3, stride=1, padding=1) if self.max_pool else _avg3(x)
        return torch.cat([self.branch1x1(x), b3, bd, self.branch_pool(p)], 1)


def resize_tf1_bilinear(x, size=299):
    """TF1 ResizeBilinear (align_corners=False, no half-pixel centres) of NCHW floats: output pixel i samples input
    coordinate i * in / out, interpolating between floor and floor + 1 (clamped at the edge)."""
    def axis(n_in, n_out, device):
        src = torch.arange(n_out, dtype=torch.float64, device=device) * (n_in / n_out)
        i0 = src.floor().long().clamp(max=n_in - 1)
        i1 = (i0 + 1).clamp(max=n_in - 1)
        return i0, i1, (src - i0.double()).float()

    N, C, H, W = x.shape
    if (H, W) == (size, size):
        return x
    y0, y1, fy = axis(H, size, x.device)
    x0, x1, fx = axis(W, size, x.device)
    top = x[:, :, y0] * (1 - fy)[:, None] + x[:, :, y1] * fy[:, None]
    return top[..., x0] * (1 - fx) + top[..., x1] * fx


class FIDInception(nn.Module):
    """pool_3 features [N, 2048] (and the 1008 logits through `fc`) of uint8 or 0..255 float images, NHWC or NCHW."""

    def __init__(self):
        super().__init__()
        self.Conv2d_1a_3x3 = Unit(3, 32, 3, stride=2)
        self.Conv2d_2a_3x3 = Unit(32, 32, 3)
        self.Conv2d_2b_3x3 = Unit(32, 64, 3, padding=1)
        self.Conv2d_3b_1x1 = Unit(64, 80, 1)
        self.Conv2d_4a_3x3 = Unit(80, 192, 3)
        self.Mixed_5b = BlockA(192, 32)
        self.Mixed_5c = BlockA(256, 64)
        self.Mixed_5d = BlockA(288, 64)
        self.Mixed_6a = BlockB(288)
        self.Mixed_6b = BlockC(768, 128)
        self.Mixed_6c = BlockC(768, 160)
        self.Mixed_6d = BlockC(768, 160)
        self.Mixed_6e = BlockC(768, 192)
        self.Mixed_7a = BlockD(768)
        self.Mixed_7b = BlockE(1280)
        self.Mixed_7c = BlockE(2048, max_pool=True)
        self.fc = nn.Linear(2048, 1008)
        self.loaded = False

    @classmethod
    def from_file(cls, path=None, map_location="cpu"):
        """The network with the published port's weights (a state dict); path defaults to GPIC_INCEPTION_WEIGHTS."""
        path = path or os.environ.get("GPIC_INCEPTION_WEIGHTS")
        if not path or not os.path.exists(path):
            raise FileNotFoundError("TF-Inception weights (pt_inception-2015-12-05 state dict) not found: pass the "
                                    "file or set GPIC_INCEPTION_WEIGHTS")
        net = cls()
        net.load_state_dict(torch.load(path, map_location=map_location, weights_only=True), strict=True)
        net.loaded = True
        return net.eval()

    @staticmethod
    def prepare(images):
        """uint8 / float 0..255 images [N, H, W, 3] or [N, 3, H, W] -> the graph's input [N, 3, 299, 299]."""
        x = images if torch.is_tensor(images) else torch.as_tensor(images)
        if x.shape[-1] == 3 and x.shape[1] != 3:
            x = x.permute(0, 3, 1, 2)
        x = resize_tf1_bilinear(x.float(), 299)
        return (x - 128.0) / 128.0

    def features(self, x):
        x = self.Conv2d_2b_3x3(self.Conv2d_2a_3x3(self.Conv2d_1a_3x3(x)))
        x = F.max_pool2d(x, 3, stride=2)
        x = self.Conv2d_4a_3x3(self.Conv2d_3b_1x1(x))
        x = F.max_pool2d(x, 3, stride=2)
        for blk in (self.Mixed_5b, self.Mixed_5c, self.Mixed_5d, self.Mixed_6a, self.Mixed_6b, self.Mixed_6c,
                    self.Mixed_6d, self.Mixed_6e, self.Mixed_7a, self.Mixed_7b, self.Mixed_7c):
            x = blk(x)
        return F.adaptive_avg_pool2d(x, 1).flatten(1)

    @torch.no_grad()
    def forward(self, images):
        return self.features(self.prepare(images).to(next(self.parameters()).device))
