"""Seeded synthetic attention inputs with the shapes and value distributions of the
benchmark configurations.

There is no public dataset for this path: the inputs are video-DiT-like q/k/v made
from a smooth Gaussian field plus white noise.

    smooth()  an N(0,1) field of shape [B*H*D, T_grid, H_grid, W_grid], blurred by a
              separable Gaussian (sigma per axis, radius ceil(3*sigma), replicate
              padding), flattened to tokens in row-major (t, h, w) order, then
              renormalised to zero mean / unit variance per (b, h, d) channel.
    Q, K      (0.5 * smooth() + 0.5 * N(0,1)) * 2 * D**-0.25, cast to bf16.
    V         N(0,1), cast to bf16.

Q, K and V are drawn in that order from one ``torch.Generator`` seeded per config.
The same code runs on CPU (parity fixtures) and on CUDA (benchmark inputs); the two
devices' generators produce different streams, so a fixture and a bench input with
the same seed are not the same tensor.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class Config:
    name: str
    batch: int
    heads: int
    head_dim: int
    grid: tuple            # (frames, height, width); tokens = prod(grid)
    block: int
    tau: float
    sigma: tuple           # blur sigma per (t, h, w) axis, in tokens
    seed: int
    taus: tuple = field(default=())

    @property
    def tokens(self) -> int:
        return self.grid[0] * self.grid[1] * self.grid[2]

    @property
    def blocks(self) -> int:
        return -(-self.tokens // self.block)

    def dense_flops(self) -> float:
        """4*B*H*T^2*D: the flops of dense attention on this shape."""
        return 4.0 * self.batch * self.heads * self.tokens ** 2 * self.head_dim


# The five configurations of the headline metric. Config 1 is the CPU-plumbing case
# (below the override's D/T gates, so the kernel API is called directly).
CONFIGS = {
    "c1": Config("c1_plumbing", 1, 2, 64, (2, 16, 16), 64, 0.9, (3.0, 3.0, 3.0), 0),
    "c2": Config("c2_image_dit", 1, 24, 128, (1, 64, 64), 128, 0.9, (3.0, 3.0, 3.0), 1),
    "c3": Config("c3_video480p", 1, 40, 128, (21, 30, 52), 128, 0.9, (1.0, 3.0, 3.0), 2),
    "c4": Config("c4_video720p", 1, 40, 128, (21, 45, 80), 128, 0.9, (1.0, 4.0, 4.0), 3,
                 taus=(0.8, 0.9, 0.95)),
    # sigma is not given for config 5; (1, 4, 4) as in config 4.
    "c5": Config("c5_long", 1, 40, 128, (31, 45, 80), 128, 0.9, (1.0, 4.0, 4.0), 4),
}


def _gaussian_taps(sigma: float, device) -> torch.Tensor:
    radius = int(math.ceil(3.0 * sigma))
    x = torch.arange(-radius, radius + 1, dtype=torch.float64)
    w = torch.exp(-(x * x) / (2.0 * sigma * sigma))
    return (w / w.sum()).to(torch.float32).to(device)


def _blur(field: torch.Tensor, sigma: tuple) -> torch.Tensor:
    """Separable Gaussian blur of [C, Tg, Hg, Wg] along the last three axes."""
    out = field.unsqueeze(1)                                    # [C, 1, Tg, Hg, Wg]
    for axis, s in enumerate(sigma):
        if s <= 0:
            continue
        taps = _gaussian_taps(float(s), field.device)
        r = (taps.numel() - 1) // 2
        shape = [1, 1, 1, 1, 1]
        shape[2 + axis] = taps.numel()
        pad = [0, 0, 0, 0, 0, 0]                                 # (w0, w1, h0, h1, t0, t1)
        pad[2 * (2 - axis)] = r
        pad[2 * (2 - axis) + 1] = r
        out = F.conv3d(F.pad(out, pad, mode="replicate"), taps.reshape(shape))
    return out.squeeze(1)


def _smooth(gen, batch, heads, dim, grid, sigma, device) -> torch.Tensor:
    channels = batch * heads * dim
    field0 = torch.randn((channels,) + tuple(grid), generator=gen, device=device,
                         dtype=torch.float32)
    blurred = _blur(field0, sigma).reshape(channels, -1)        # [C, T] row-major (t,h,w)
    mean = blurred.mean(dim=1, keepdim=True)
    std = blurred.var(dim=1, unbiased=False, keepdim=True).clamp_min(1e-12).sqrt()
    blurred = (blurred - mean) / std
    tokens = blurred.shape[1]
    return blurred.reshape(batch, heads, dim, tokens).permute(0, 3, 1, 2)   # BTHD


def make_qkv(cfg: Config, device="cpu", heads=None):
    """(q, k, v) bf16 [B, T, H, D] for ``cfg``; ``heads`` (a slice) keeps a head range
    of the full draw, so a head slice is bit-identical to the same heads of the full
    tensors."""
    gen = torch.Generator(device=device)
    gen.manual_seed(cfg.seed)
    B, H, D, grid = cfg.batch, cfg.heads, cfg.head_dim, cfg.grid
    T = cfg.tokens
    amp = 2.0 * D ** -0.25
    out = []
    for _ in range(2):
        s = _smooth(gen, B, H, D, grid, cfg.sigma, device)
        n = torch.randn((B, T, H, D), generator=gen, device=device, dtype=torch.float32)
        out.append(((0.5 * s + 0.5 * n) * amp).to(torch.bfloat16).contiguous())
        del s, n
    v = torch.randn((B, T, H, D), generator=gen, device=device,
                    dtype=torch.float32).to(torch.bfloat16)
    q, k = out
    if heads is not None:
        q, k, v = (t[:, :, heads].contiguous() for t in (q, k, v))
    return q, k, v


def custom_config(name, batch, heads, head_dim, grid, block, tau, sigma, seed):
    return Config(name, batch, heads, head_dim, tuple(grid), block, tau, tuple(sigma), seed)
