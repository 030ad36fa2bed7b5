"""Pixel-space "autoencoder": the identity up to an affine scale/shift, so the denoiser works on pixels
(reference baselines/PixelGen/src/models/autoencoder/pixel.py, base.py). uint8 <-> float helpers with the reference's
rounding."""
import torch


class BaseAE(torch.nn.Module):
    def __init__(self, scale=1.0, shift=0.0):
        super().__init__()
        self.scale, self.shift = scale, shift

    def encode(self, x):
        return self._impl_encode(x)

    def decode(self, x):
        return self._impl_decode(x)

    def _impl_encode(self, x):
        raise NotImplementedError

    def _impl_decode(self, x):
        raise NotImplementedError


class PixelAE(BaseAE):
    """encode(x) = x / scale + shift; decode(z) = (z - shift) * scale."""

    def _impl_encode(self, x):
        return x / self.scale + self.shift

    def _impl_decode(self, x):
        return (x - self.shift) * self.scale


def uint82fp(x):
    """uint8 [0, 255] -> float32 [-1, 1]."""
    return (x.to(torch.float32) - 127.5) / 127.5


def fp2uint8(x):
    """[-1, 1] floats -> uint8, rounded half up and clipped."""
    return torch.clip_((x + 1) * 127.5 + 0.5, 0, 255).to(torch.uint8)
