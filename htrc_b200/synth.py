"""Seeded synthetic Q/K/V for the flat HTRC workloads (the reference's real captures are private).

Video-latent inputs (configurations 2-4 of the benchmark): per channel of each head, N(0, 1) on a
coarse 4 x 8 x 8 (t, h, w) grid, trilinearly upsampled (align_corners=False) to the latent grid,
plus 0.5 * N(0, 1) noise, flattened row-major over (t, h, w) and rescaled so that the head's RMS is
3.  Q and K are independent draws, V ~ N(0, 1); all three are returned as bfloat16 [N, D].
Seeds: ``base + 1000 * block + 100 * batch + head`` (one CPU torch.Generator per head), so any
(block, batch, head) can be regenerated alone, on any machine.

The fallback generator of the reference's sweep tool (low-rank mix + noise,
tools/sweep_h3_flat_kernels.py:185-194) is provided as ``lowrank_inputs`` for small tests.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

GRID_SMALL = (16, 32, 32)      # 16,384 tokens
GRID_FULL = (32, 48, 84)       # 129,024 tokens (1344 x 768, 124 frames)
GRID_243 = (61, 48, 84)        # 245,952 tokens


def _field(gen, grid, d, rms):
    t, h, w = grid
    base = torch.randn((1, d, 4, 8, 8), generator=gen, dtype=torch.float32)
    up = F.interpolate(base, size=(t, h, w), mode="trilinear", align_corners=False)[0]
    x = up.reshape(d, t * h * w).T.contiguous()
    x += 0.5 * torch.randn((t * h * w, d), generator=gen, dtype=torch.float32)
    x *= rms / x.pow(2).mean().sqrt()
    return x


def head_inputs(grid=GRID_FULL, d=128, *, head=0, batch=0, block=0, base_seed=0, rms=3.0,
                dtype=torch.bfloat16):
    """(q, k, v) of one head on the CPU, each [t*h*w, d] in ``dtype``."""
    gen = torch.Generator().manual_seed(int(base_seed) + 1000 * int(block) + 100 * int(batch) + int(head))
    q = _field(gen, grid, d, rms)
    k = _field(gen, grid, d, rms)
    n = q.shape[0]
    v = torch.randn((n, d), generator=gen, dtype=torch.float32)
    return q.to(dtype), k.to(dtype), v.to(dtype)


def cluster_inputs(n=4096, d=64, *, clusters=64, swap=0.1, sigma=0.3, centre_std=2.0, seed=0):
    """Configuration 1 of the benchmark (the CPU NumPy case), float32 NumPy arrays (q, k, v), each [n, d]:
    ``clusters`` centres ~ N(0, centre_std^2 I); token i belongs to cluster i // (n / clusters) except a
    ``swap`` fraction of tokens whose cluster is redrawn uniformly; q and k = centre + sigma * N(0, 1)
    (independent memberships and noise), v ~ N(0, 1).  Seeded ``numpy.random.default_rng(seed)``."""
    import numpy as np
    rng = np.random.default_rng(int(seed))
    cen = rng.standard_normal((clusters, d)) * centre_std
    per = max(1, n // clusters)

    def members():
        ids = np.minimum(np.arange(n) // per, clusters - 1)
        sw = rng.random(n) < swap
        ids[sw] = rng.integers(0, clusters, int(sw.sum()))
        return ids

    q = cen[members()] + sigma * rng.standard_normal((n, d))
    k = cen[members()] + sigma * rng.standard_normal((n, d))
    v = rng.standard_normal((n, d))
    return q.astype(np.float32), k.astype(np.float32), v.astype(np.float32)


def lowrank_inputs(n, m, d=128, *, seed=1234, rank=24, noise=0.6, dtype=torch.bfloat16):
    """Low-rank mix + noise keys/queries, N(0, 1) values (CPU)."""
    gen = torch.Generator().manual_seed(int(seed))
    basis = torch.randn((rank, d), generator=gen)

    def mix(rows):
        c = torch.randn((rows, rank), generator=gen) * 0.45
        return c @ basis + noise * torch.randn((rows, d), generator=gen)

    q = mix(n)
    k = mix(m)
    v = torch.randn((m, d), generator=gen)
    return q.to(dtype), k.to(dtype), v.to(dtype)
