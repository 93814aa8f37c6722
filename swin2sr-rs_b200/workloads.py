"""The five configurations BASELINE.json names, as seeded synthetic workloads.

Weights: ``weights.Weights.seeded(task, 0)`` (the published init distributions
from a numpy seed). Inputs follow the recipes fixed for the build (seeded torch
generators, so every machine regenerates the same tensors):

* LW  lightweight-x2, one 64x64 image, ``torch.rand`` seed 1;
* C2  classical-x2, one 256x256 image, seed 1;
* C4  classical-x4, one 240x320 smooth field: per channel, 8 sinusoids with
      amplitude U(0.05, 0.20), frequencies U(0.5, 8) cycles per image and phase
      U(0, 2pi), ``clip(0.5 + sum, 0, 1)``, generator seed 3;
* RW  realworld-x4, one 512x512 image, seed 4, plus a per-8x8-block, per-channel
      offset U(-4/255, 4/255) from the same generator, clipped to [0, 1];
* CX  compressed-x4, a batch of 256 48x48 images, seed 7.
"""
from __future__ import annotations

import math

import numpy as np

WORKLOADS = {
    "lightweight-x2": dict(task="lightweight_sr", batch=1, h=64, w=64),
    "classical-x2": dict(task="classical_sr_x2", batch=1, h=256, w=256),
    "classical-x4": dict(task="classical_sr", batch=1, h=240, w=320),
    "realworld-x4": dict(task="real_sr", batch=1, h=512, w=512),
    "compressed-x4": dict(task="compressed_sr", batch=256, h=48, w=48),
}


def make_input(name: str, batch: int | None = None) -> np.ndarray:
    """[B][3][h][w] float32 in [0, 1] for workload ``name``."""
    import torch

    wl = WORKLOADS[name]
    B = batch or wl["batch"]
    h, w = wl["h"], wl["w"]
    if name in ("lightweight-x2", "classical-x2"):
        g = torch.Generator().manual_seed(1)
        return torch.rand(B, 3, h, w, generator=g).numpy()
    if name == "compressed-x4":
        g = torch.Generator().manual_seed(7)
        return torch.rand(B, 3, h, w, generator=g).numpy()
    if name == "realworld-x4":
        g = torch.Generator().manual_seed(4)
        x = torch.rand(B, 3, h, w, generator=g)
        off = (torch.rand(B, 3, h // 8, w // 8, generator=g) * 2 - 1) * (4.0 / 255.0)
        x = x + off.repeat_interleave(8, dim=2).repeat_interleave(8, dim=3)
        return x.clamp(0, 1).numpy()
    if name == "classical-x4":
        g = torch.Generator().manual_seed(3)
        yy = torch.arange(h, dtype=torch.float64)[:, None] / h
        xx = torch.arange(w, dtype=torch.float64)[None, :] / w
        out = torch.empty(B, 3, h, w, dtype=torch.float64)
        for b in range(B):
            for c in range(3):
                acc = torch.full((h, w), 0.5, dtype=torch.float64)
                for _ in range(8):
                    r = torch.rand(4, generator=g, dtype=torch.float64)
                    a = 0.05 + 0.15 * r[0]
                    fy = 0.5 + 7.5 * r[1]
                    fx = 0.5 + 7.5 * r[2]
                    ph = 2 * math.pi * r[3]
                    acc += a * torch.sin(2 * math.pi * (fy * yy + fx * xx) + ph)
                out[b, c] = acc.clamp(0, 1)
        return out.float().numpy()
    raise KeyError(name)


def batch_shard(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Images [lo, hi) of a batch that rank ``rank`` of ``world`` runs in the batch
    data-parallel mode: contiguous, equal shards in rank order, so the ranks' outputs
    concatenate to the batch's. The images are independent (no exchange); a batch
    that does not divide evenly is refused, so every rank times the same work."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if batch % world:
        raise ValueError(f"batch {batch} does not split over {world} ranks")
    n = batch // world
    return rank * n, (rank + 1) * n


def adjust(x: np.ndarray, wt) -> np.ndarray:
    """Pre::adjust over a batch: (x - mean) * img_range (src/backend.rs:76-86)."""
    m = np.asarray(wt.mean, np.float32)[None, :, None, None]
    return ((x - m) * np.float32(wt.img_range)).astype(np.float32)
