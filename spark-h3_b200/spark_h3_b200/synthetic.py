"""Seeded synthetic Q/K/V with the shapes and value structure of the benchmark configs.

Each tensor is a sum of 8 low-frequency 3-D sinusoids over the (t, h, w) video grid in
THW raster order (integer frequencies in [0, 2]^3, uniform phases, a direction with
unit-variance N(0, 1) entries per sinusoid, amplitude 1.0) plus 0.3 * N(0, 1) noise.
The clustered variant adds one of 64 N(0, 1) centroids per spatial region (a 4x4x4
partition of the grid) with 0.25 * N(0, 1) noise.  Tensors are BTHD.
"""
from __future__ import annotations

import math

import torch


def grid_positions(grid: tuple[int, int, int], device=None) -> torch.Tensor:
    """Normalised (t, h, w) coordinates in [0, 1) of every token, THW raster order."""
    t, h, w = grid
    tt, hh, ww = torch.meshgrid(
        torch.arange(t, device=device, dtype=torch.float32) / t,
        torch.arange(h, device=device, dtype=torch.float32) / h,
        torch.arange(w, device=device, dtype=torch.float32) / w,
        indexing="ij",
    )
    return torch.stack((tt, hh, ww), dim=-1).reshape(-1, 3)


def sinusoid_tensor(grid, heads: int, head_dim: int, *, generator: torch.Generator, device=None,
                    dtype=torch.float32, noise: float = 0.3, clustered: bool = False,
                    chunk: int = 16384) -> torch.Tensor:
    pos = grid_positions(grid, device)
    n = pos.shape[0]
    width = heads * head_dim
    freqs = torch.randint(0, 3, (8, 3), generator=generator, device=device).to(torch.float32)
    phase = torch.rand(8, generator=generator, device=device) * (2 * math.pi)
    direction = torch.randn(8, width, generator=generator, device=device)
    centroids = region = None
    if clustered:
        centroids = torch.randn(64, width, generator=generator, device=device)
        cell = (pos * 4).floor().clamp(max=3).to(torch.int64)
        region = cell[:, 0] * 16 + cell[:, 1] * 4 + cell[:, 2]
        noise = 0.25
    out = torch.empty((n, width), device=device, dtype=dtype)
    for start in range(0, n, chunk):
        stop = min(n, start + chunk)
        feat = torch.sin(2 * math.pi * (pos[start:stop] @ freqs.T) + phase)
        x = feat @ direction
        x += noise * torch.randn(stop - start, width, generator=generator, device=device)
        if clustered:
            x += centroids[region[start:stop]]
        out[start:stop] = x.to(dtype)
    return out.view(1, n, heads, head_dim)


def make_qkv(grid, heads: int, head_dim: int, *, seed: int = 0, device=None, dtype=torch.bfloat16,
             q_scale: float = 1.0, clustered: bool = False, with_v: bool = True):
    """Q, K, V [1, T, H, D]; Q is multiplied by q_scale (config 1 uses 1/sqrt(D)).  With
    with_v=False only Q and K are drawn (V is drawn last, so Q and K are the same)."""
    gen = torch.Generator(device=device if device is not None else "cpu").manual_seed(seed)
    q = sinusoid_tensor(grid, heads, head_dim, generator=gen, device=device, clustered=clustered)
    if q_scale != 1.0:
        q.mul_(q_scale)
    q = q.to(dtype)
    k = sinusoid_tensor(grid, heads, head_dim, generator=gen, device=device, dtype=dtype, clustered=clustered)
    if not with_v:
        return q, k
    v = sinusoid_tensor(grid, heads, head_dim, generator=gen, device=device, dtype=dtype, clustered=clustered)
    return q, k, v


# Benchmark configurations.
CONFIGS = {
    0: dict(grid=(4, 32, 32), heads=4, head_dim=64, dtype=torch.float32, block=64, topk_ratio=0.1,
            q_scale=1.0, mode="reweight_only"),
    1: dict(grid=(31, 48, 84), heads=32, head_dim=128, dtype=torch.bfloat16, block=128, topk_ratio=0.1,
            q_scale=128 ** -0.5, mode="reweight_only"),
    2: dict(grid=(61, 48, 84), heads=32, head_dim=128, dtype=torch.bfloat16, block=64, topk_ratio=0.1,
            q_scale=1.0, mode="full", clustered=True),
}
