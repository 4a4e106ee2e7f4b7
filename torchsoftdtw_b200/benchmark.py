"""Benchmark sweep of the SoftDTW module on CUDA: ``python -m torchsoftdtw_b200.benchmark``.

The grid follows the reference's own sweep (``src/torchsoftdtw/benchmark/run_benchmark.py:35-41``: batch
size, padded length and feature size from short/large-batch to long/small-batch workloads, gamma = 1) and
its length spreads (``generate.py:19-22``: every sample at the padded length, lengths drawn from
[0.9 L, L], or from [0.25 L, L], frames past a sample's length zeroed). The reference's sweep compares
third-party implementations; this one times this package's module alone, forward and forward + backward
(loss = costs.sum(), gradient w.r.t. X), with CUDA events after a warm-up, and reports the time per call
and the DP cells per second (cells = in-range cells of every pair, counted exactly).

    python -m torchsoftdtw_b200.benchmark [--min-time 0.2] [--forward-only] [--distance l2_squared|l1|cosine]
                                          [--grid sweep|headline] [--gamma 1.0] [--unfused] [--output FILE]

``--grid headline`` times the single headline workload (B=256, L=512, D=64, every sample full length);
``--unfused`` also times the composition a user of the reference runs (the distance's torch expression
for D, then ``soft_dtw`` and torch autograd through the expression).
"""

from __future__ import annotations

import argparse
import statistics
import sys

import torch

GAMMA = 1.0
SEED = 0
# (batch size, padded length, feature size)
GRID = [(64, 16, 8), (64, 64, 8), (64, 256, 12), (32, 256, 16), (16, 512, 16)]
GRIDS = {"sweep": GRID, "headline": [(256, 512, 64)]}
# lower end of the drawn lengths, as a fraction of the padded length
SPREADS = {"none": 1.0, "small": 0.9, "large": 0.25}


def make_batch(batch: int, length: int, feat: int, spread: str, device: torch.device, seed: int = SEED):
    """Seeded N(0, 1) sequences of `length` padded frames; per-sample lengths drawn for `spread`, frames
    past a sample's length set to zero."""
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(batch, length, feat, generator=g)
    Y = torch.randn(batch, length, feat, generator=g)
    lo = SPREADS[spread]
    if lo >= 1.0:
        lx = torch.full((batch,), length, dtype=torch.long)
        ly = torch.full((batch,), length, dtype=torch.long)
    else:
        first = max(1, round(lo * length))
        lx = torch.randint(first, length + 1, (batch,), generator=g)
        ly = torch.randint(first, length + 1, (batch,), generator=g)
    frame = torch.arange(length)
    X[frame[None, :] >= lx[:, None]] = 0.0
    Y[frame[None, :] >= ly[:, None]] = 0.0
    return X.to(device), Y.to(device), lx.to(device), ly.to(device)


def time_call(fn, min_time: float) -> float:
    """Median milliseconds of `fn` over CUDA-event timed calls, at least `min_time` seconds of them."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    samples: list[float] = []
    total = 0.0
    while total < min_time * 1e3 or len(samples) < 10:
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ms = a.elapsed_time(b)
        samples.append(ms)
        total += ms
    return statistics.median(samples)


def run(min_time: float = 0.2, forward_only: bool = False, distance: str = "l2_squared", grid: str = "sweep",
        gamma: float = GAMMA, unfused: bool = False) -> list[dict]:
    import torchsoftdtw_b200 as T
    from torchsoftdtw_b200.distances import PAIRWISE_DISTANCES

    dev = torch.device("cuda", torch.cuda.current_device())
    module = T.SoftDTW(gamma=gamma, distance=distance)
    expr = PAIRWISE_DISTANCES[distance]
    rows = []
    for batch, length, feat in GRIDS[grid]:
        for spread in (SPREADS if grid == "sweep" else ["none"]):
            X, Y, lx, ly = make_batch(batch, length, feat, spread, dev)
            cells = float((lx * ly).sum().item())
            row = {"B": batch, "L": length, "D": feat, "spread": spread, "cells": cells}
            row["fwd_ms"] = time_call(lambda: module(X, Y, lx, ly), min_time)
            if not forward_only:
                Xg = X.clone().requires_grad_(True)

                def step():
                    Xg.grad = None
                    module(Xg, Y, lx, ly).sum().backward()

                row["fwdbwd_ms"] = time_call(step, min_time)
                if unfused:
                    def step_unfused():
                        Xg.grad = None
                        T.soft_dtw(expr(Xg, Y), lx, ly, gamma).sum().backward()

                    row["unfused_fwdbwd_ms"] = time_call(step_unfused, min_time)
            T.check_errors(dev)
            rows.append(row)
    return rows


def table(rows: list[dict], device_name: str, distance: str = "l2_squared", gamma: float = GAMMA) -> str:
    has_bwd = "fwdbwd_ms" in rows[0]
    has_unf = "unfused_fwdbwd_ms" in rows[0]
    head = f"SoftDTW module, {device_name}, gamma = {gamma}, distance = {distance}, fp32\n\n"
    cols = "| B | L | D | spread | fwd ms | fwd cells/s |" + (" fwd+bwd ms | fwd+bwd cells/s |" if has_bwd else "")
    cols += " unfused fwd+bwd ms |" if has_unf else ""
    sep = "|---|---|---|---|---|---|" + ("---|---|" if has_bwd else "") + ("---|" if has_unf else "")
    lines = [head + cols, sep]
    for r in rows:
        line = (f"| {r['B']} | {r['L']} | {r['D']} | {r['spread']} | {r['fwd_ms']:.3f} | "
                f"{r['cells'] / (r['fwd_ms'] / 1e3):.3e} |")
        if has_bwd:
            line += f" {r['fwdbwd_ms']:.3f} | {r['cells'] / (r['fwdbwd_ms'] / 1e3):.3e} |"
        if has_unf:
            line += f" {r['unfused_fwdbwd_ms']:.3f} |"
        lines.append(line)
    return "\n".join(lines) + "\n"


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--min-time", type=float, default=0.2, help="seconds of timed calls per measurement")
    ap.add_argument("--forward-only", action="store_true")
    ap.add_argument("--distance", default="l2_squared", choices=["l2_squared", "l1", "cosine"])
    ap.add_argument("--grid", default="sweep", choices=list(GRIDS))
    ap.add_argument("--gamma", type=float, default=GAMMA)
    ap.add_argument("--unfused", action="store_true", help="also time the unfused composition")
    ap.add_argument("--output", default=None, help="also write the table to this file")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        print("torchsoftdtw_b200.benchmark needs a CUDA device", file=sys.stderr)
        return 1
    rows = run(args.min_time, args.forward_only, args.distance, args.grid, args.gamma, args.unfused)
    text = table(rows, torch.cuda.get_device_name(), args.distance, args.gamma)
    print(text)
    if args.output:
        with open(args.output, "w") as f:
            f.write(text)
    return 0


if __name__ == "__main__":
    sys.exit(main())
