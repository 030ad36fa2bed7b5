"""Fixed tables and small modules of JiT-T2I, written from the reference's formulas.

* rope_tables: 2D RoPE angles of baselines/PixelGen/src/models/layers/rope.py:22-37 (precompute_freqs_cis_ex2d with
  scale 1): positions linspace(0, H, W) in x and linspace(0, W, H) in y on a row-major grid, frequencies
  theta^(-4k/dim) for k < dim/4, pairs interleaved (x, y) -> [N, dim/2] cos and sin tables (fp32).
* sincos_pos_embed: fixed 2D sin-cos table of JiT_T2I.py:78-111 (half the channels encode the grid's w coordinate
  first, then h; each half is [sin | cos] with omega = 1 / 10000^(2i / (D/2))).
* timestep_freq: the TimestepEmbedder's frequency features (baselines/PixelGen/src/models/layers/time_embed.py:16-24)
  with max_period = 10: [cos(t f_k), sin(t f_k)], f_k = exp(-ln(10) k / half).
"""
import math

import numpy as np
import torch
import torch.nn as nn


def rope_tables(head_dim, height, width, theta=10000.0, scale=1.0, device=None):
    x_pos = torch.linspace(0, height * scale, width)
    y_pos = torch.linspace(0, width * scale, height)
    y_pos, x_pos = torch.meshgrid(y_pos, x_pos, indexing="ij")
    y_pos, x_pos = y_pos.reshape(-1), x_pos.reshape(-1)
    freqs = 1.0 / (theta ** (torch.arange(0, head_dim, 4)[: head_dim // 4].float() / head_dim))
    xa = torch.outer(x_pos, freqs).float()
    ya = torch.outer(y_pos, freqs).float()
    ang = torch.stack([xa, ya], dim=-1).reshape(height * width, -1)  # interleaved x, y -> [N, head_dim / 2]
    # the reference builds the table with torch.polar in fp32; cos/sin of the same fp32 angles
    cis = torch.polar(torch.ones_like(ang), ang)
    cos, sin = cis.real.contiguous().float(), cis.imag.contiguous().float()
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos, sin


def _sincos_1d(dim, pos):
    omega = np.arange(dim // 2, dtype=np.float64)
    omega /= dim / 2.0
    omega = 1.0 / 10000 ** omega
    out = np.einsum("m,d->md", pos.reshape(-1), omega)
    return np.concatenate([np.sin(out), np.cos(out)], axis=1)


def sincos_pos_embed(dim, grid_size):
    gh = np.arange(grid_size, dtype=np.float32)
    gw = np.arange(grid_size, dtype=np.float32)
    grid = np.stack(np.meshgrid(gw, gh), axis=0).reshape(2, 1, grid_size, grid_size)
    emb = np.concatenate([_sincos_1d(dim // 2, grid[0]), _sincos_1d(dim // 2, grid[1])], axis=1)
    return torch.from_numpy(emb).float()


def timestep_freq(t, dim=256, max_period=10):
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(0, half, dtype=torch.float32, device=t.device) / half)
    args = t[..., None].float() * freqs[None]
    emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
    if dim % 2:
        emb = torch.cat([emb, torch.zeros_like(emb[:, :1])], dim=-1)
    return emb


class RMSNorm(nn.Module):
    """Parameter holder with the reference's name (`weight`) and epsilon attribute (`variance_epsilon`)."""

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.variance_epsilon = eps


class Linear(nn.Module):
    """nn.Linear's parameters (`weight` [out, in], optional `bias`) without its forward: the blocks run the fused ops."""

    def __init__(self, fan_in, fan_out, bias=True):
        super().__init__()
        self.in_features, self.out_features = fan_in, fan_out
        self.weight = nn.Parameter(torch.empty(fan_out, fan_in))
        self.bias = nn.Parameter(torch.empty(fan_out)) if bias else None

    def extra_repr(self):
        return f"in={self.in_features}, out={self.out_features}, bias={self.bias is not None}"
