"""Seeded synthetic inputs for the five Soft-DTW workloads this library is measured and tested on.

No public dataset is involved; each workload is generated from one CPU ``torch.Generator`` seeded with
``seed`` (inputs X, then Y, then lengths, in that order), so every process and every rank sees the same
global batch. ``batch`` overrides B (a prefix-compatible smaller draw is NOT guaranteed: it is a fresh
draw of the smaller shape).

=========  ==============================================================================================
readme     X (8,50,16), Y (8,40,16) fp32 ~ N(0,1); gamma=1, normalize, no band, full lengths
medium     X, Y (256,512,64) fp32 ~ N(0,1); gamma=0.1, no band  (the headline throughput workload)
ragged     X (512,256,32), Y (512,192,32) fp32 random walks (cumsum of N(0, 0.1^2) steps);
           lengths_x ~ U{64..256}, lengths_y ~ U{48..192}; bandwidth 32; gamma=0.5; normalize
long       X, Y (16,4096,128) fp32 sin(2 pi f t + phi) + N(0, 0.05^2), f ~ U[0.001,0.02],
           phi ~ U[0, 2 pi) per (b, channel); bandwidth 256; gamma=0.01
largebatch X, Y (65536,64,4) fp64 ~ U[-1,1]; gamma=1, no band
=========  ==============================================================================================
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    N: int
    M: int
    d: int
    dtype: torch.dtype
    gamma: float
    bandwidth: int
    normalize: bool
    kind: str  # "normal" | "randwalk" | "sine" | "uniform"
    ragged: tuple[int, int, int, int] | None = None  # (lx_lo, lx_hi, ly_lo, ly_hi), inclusive


WORKLOADS: dict[str, Workload] = {
    "readme": Workload("readme", 8, 50, 40, 16, torch.float32, 1.0, -1, True, "normal"),
    "medium": Workload("medium", 256, 512, 512, 64, torch.float32, 0.1, -1, False, "normal"),
    "ragged": Workload("ragged", 512, 256, 192, 32, torch.float32, 0.5, 32, True, "randwalk", (64, 256, 48, 192)),
    "long": Workload("long", 16, 4096, 4096, 128, torch.float32, 0.01, 256, False, "sine"),
    "largebatch": Workload("largebatch", 65536, 64, 64, 4, torch.float64, 1.0, -1, False, "uniform"),
}


def _series(g: torch.Generator, kind: str, B: int, T: int, d: int, dtype: torch.dtype) -> torch.Tensor:
    if kind == "normal":
        return torch.randn(B, T, d, generator=g, dtype=torch.float64).to(dtype)
    if kind == "uniform":
        return (torch.rand(B, T, d, generator=g, dtype=torch.float64) * 2 - 1).to(dtype)
    if kind == "randwalk":
        steps = torch.randn(B, T, d, generator=g, dtype=torch.float64) * 0.1
        return steps.cumsum(dim=1).to(dtype)
    if kind == "sine":
        f = 0.001 + torch.rand(B, 1, d, generator=g, dtype=torch.float64) * (0.02 - 0.001)
        phi = torch.rand(B, 1, d, generator=g, dtype=torch.float64) * (2 * math.pi)
        t = torch.arange(T, dtype=torch.float64).view(1, T, 1)
        noise = torch.randn(B, T, d, generator=g, dtype=torch.float64) * 0.05
        return (torch.sin(2 * math.pi * f * t + phi) + noise).to(dtype)
    raise ValueError(kind)


def make_inputs(name: str, seed: int = 0, batch: int | None = None, N: int | None = None, M: int | None = None,
                d: int | None = None):
    """Returns (X, Y, lengths_x, lengths_y, workload) on the CPU; lengths are int64 (B,)."""
    w = WORKLOADS[name]
    B = batch if batch is not None else w.B
    N_ = N if N is not None else w.N
    M_ = M if M is not None else w.M
    d_ = d if d is not None else w.d
    g = torch.Generator(device="cpu").manual_seed(seed)
    X = _series(g, w.kind, B, N_, d_, w.dtype)
    Y = _series(g, w.kind, B, M_, d_, w.dtype)
    if w.ragged is not None:
        lo_x, hi_x, lo_y, hi_y = w.ragged
        hi_x, hi_y = min(hi_x, N_), min(hi_y, M_)
        lo_x, lo_y = min(lo_x, hi_x), min(lo_y, hi_y)
        lx = torch.randint(lo_x, hi_x + 1, (B,), generator=g, dtype=torch.int64)
        ly = torch.randint(lo_y, hi_y + 1, (B,), generator=g, dtype=torch.int64)
    else:
        lx = torch.full((B,), N_, dtype=torch.int64)
        ly = torch.full((B,), M_, dtype=torch.int64)
    return X, Y, lx, ly, w


def count_cells(lengths_x: torch.Tensor, lengths_y: torch.Tensor, bandwidth: int) -> int:
    """Exact number of DP cells (in-band, inside the lengths) of a batch, by the band's row intervals."""
    from ._ext import capi

    lib = capi()
    pairs: dict[tuple[int, int], int] = {}
    total = 0
    for nx, ny in zip(lengths_x.tolist(), lengths_y.tolist()):
        key = (int(nx), int(ny))
        if key not in pairs:
            pairs[key] = int(lib.sdtw_pair_cells(key[0], key[1], int(bandwidth)))
        total += pairs[key]
    return total
