"""Generates the golden fixtures of tests/golden/ by running the REFERENCE itself (run only where the
reference sources are mounted; the committed .npz files are what the tests read everywhere else).

* op-level cases: the reference's CPU operator compiled from its own source file (oracle/_ref, built by
  ``make -C oracle ref``), called through its schemas ``torch.ops.torchsoftdtw_ref.forward/backward``;
* module-level cases: the reference's own ``distances.pairwise_l2_squared`` (imported from the reference
  source tree) composed with that operator under torch autograd, exactly as the reference's
  ``SoftDTW.forward`` does (``softdtw.py:106-142``): costs, optional normalize, grad_X and grad_Y of
  ``costs.sum()``.

Usage: python tests/golden/make_golden.py [--ref-root /root/reference]
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from torchsoftdtw_b200.workloads import make_inputs  # noqa: E402

GAMMA_SWEEP = (0.001, 0.01, 0.1, 1, 10, 100, 1000)


def load_ref_distances(ref_root: str):
    path = os.path.join(ref_root, "src", "torchsoftdtw", "distances.py")
    spec = importlib.util.spec_from_file_location("ref_distances", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class RefAutograd(torch.autograd.Function):
    """The reference's SoftDTWAutograd (softdtw.py:33-48) over the compiled reference ops."""

    @staticmethod
    def forward(ctx, D, lx, ly, gamma, bw):
        ops = O.load_ref()
        costs, R = ops.forward(D, lx, ly, gamma, bw)
        ctx.save_for_backward(D, R, lx, ly)
        ctx.gamma, ctx.bw = gamma, bw
        return costs

    @staticmethod
    def backward(ctx, g):
        ops = O.load_ref()
        D, R, lx, ly = ctx.saved_tensors
        E = ops.backward(D, R, lx, ly, ctx.gamma, ctx.bw)
        return g.unsqueeze(-1).unsqueeze(-1) * E, None, None, None, None


def op_case(D, lx, ly, gamma, bw, keep_R=True):
    ops = O.load_ref()
    costs, R = ops.forward(D, lx, ly, gamma, bw)
    E = ops.backward(D, R, lx, ly, gamma, bw)
    out = dict(D=D.numpy(), lx=lx.numpy(), ly=ly.numpy(), gamma=np.float64(gamma), bw=np.int64(bw),
               costs=costs.numpy(), E=E.numpy())
    if keep_R:
        out["R"] = R.numpy()
    return out


def module_case(dist, X, Y, lx, ly, gamma, bw, normalize):
    X = X.clone().requires_grad_(True)
    Y = Y.clone().requires_grad_(True)
    D = dist.pairwise_l2_squared(X, Y)
    costs = RefAutograd.apply(D, lx, ly, gamma, bw)
    if normalize:
        costs = costs / (lx + ly - 1).to(costs.dtype)
    costs.sum().backward()
    return dict(X=X.detach().numpy(), Y=Y.detach().numpy(), lx=lx.numpy(), ly=ly.numpy(), gamma=np.float64(gamma),
                bw=np.int64(bw), normalize=np.bool_(normalize), costs=costs.detach().numpy(),
                grad_X=X.grad.numpy(), grad_Y=Y.grad.numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", default="/root/reference")
    args = ap.parse_args()
    if not O.ref_available():
        O.build()
    dist = load_ref_distances(args.ref_root)
    cases: dict[str, dict] = {}

    # --- op level (D given), shapes from the reference's own tests --------------------------------------
    torch.manual_seed(42)
    D = torch.rand(2, 5, 7, dtype=torch.float64)
    for g in GAMMA_SWEEP:
        cases[f"op_basic_g{g}"] = op_case(D, torch.tensor([5, 5]), torch.tensor([7, 7]), float(g), -1)
    cases["op_single"] = op_case(torch.tensor([[[2.0]]], dtype=torch.float64), torch.tensor([1]), torch.tensor([1]),
                                 1.0, -1)
    torch.manual_seed(1)
    cases["op_padding"] = op_case(torch.rand(3, 8, 8, dtype=torch.float64), torch.tensor([4, 6, 3]),
                                  torch.tensor([5, 4, 7]), 0.5, -1)
    torch.manual_seed(7)
    for N, M in [(4, 8), (8, 4), (7, 4), (5, 6), (3, 10)]:
        Dr = torch.rand(2, N, M, dtype=torch.float64)
        for bw in (0, 1, 2):
            cases[f"op_band_{N}x{M}_bw{bw}"] = op_case(Dr, torch.tensor([N, N]), torch.tensor([M, M]), 0.5, bw)
    torch.manual_seed(500)
    cases["op_band_padding"] = op_case(torch.rand(3, 10, 10, dtype=torch.float64), torch.tensor([6, 8, 5]),
                                       torch.tensor([7, 6, 9]), 0.5, 3)
    for seed, (B, N, M, g, bw) in enumerate([(4, 6, 8, 1.0, -1), (4, 6, 8, 0.5, 2), (3, 5, 5, 1.0, -1)]):
        torch.manual_seed(seed)
        Dp = torch.rand(B, N, M, dtype=torch.float64)
        lx = torch.randint(max(1, N - 3), N + 1, (B,))
        ly = torch.randint(max(1, M - 3), M + 1, (B,))
        cases[f"op_parity_{B}x{N}x{M}_bw{bw}"] = op_case(Dp, lx, ly, g, bw)
    torch.manual_seed(3)
    for N, M in [(120, 130), (150, 110), (110, 150), (130, 130)]:
        Dt = torch.rand(2, N, M, dtype=torch.float64)
        lx = torch.randint(N - 3, N + 1, (2,))
        ly = torch.randint(M - 3, M + 1, (2,))
        cases[f"op_mid_{N}x{M}"] = op_case(Dt, lx, ly, 0.7, -1, keep_R=False)
    torch.manual_seed(4)
    cases["op_mid_band50"] = op_case(torch.rand(2, 120, 130, dtype=torch.float64), torch.tensor([118, 120]),
                                     torch.tensor([130, 128]), 1.0, 50, keep_R=False)
    torch.manual_seed(6)
    cases["op_rect_150x900_bw10"] = op_case(torch.rand(1, 150, 900, dtype=torch.float64), torch.tensor([149]),
                                             torch.tensor([897]), 1.0, 10, keep_R=False)
    torch.manual_seed(11)
    Dz = torch.rand(4, 33, 65, dtype=torch.float64)
    cases["op_zero_lengths"] = op_case(Dz, torch.tensor([0, 33, 0, 1]), torch.tensor([65, 0, 0, 1]), 1.0, -1)
    for edge, shape in [("1xM", (1, 1, 5)), ("Nx1", (1, 5, 1)), ("2x20", (1, 2, 20)), ("20x2", (1, 20, 2))]:
        torch.manual_seed(300)
        De = torch.rand(*shape, dtype=torch.float64)
        cases[f"op_edge_{edge}"] = op_case(De, torch.tensor([shape[1]]), torch.tensor([shape[2]]), 0.5, -1)
    # fp32 op cases (parity of the fp32 kernels against the reference's fp32 arithmetic)
    torch.manual_seed(701)
    cases["op_f32_small"] = op_case(torch.rand(4, 37, 45, dtype=torch.float32), torch.tensor([37, 30, 12, 1]),
                                    torch.tensor([45, 44, 40, 3]), 1.0, -1)
    torch.manual_seed(702)
    cases["op_f32_band"] = op_case(torch.rand(3, 70, 50, dtype=torch.float32) * 4, torch.tensor([70, 64, 33]),
                                   torch.tensor([50, 49, 47]), 0.5, 4)

    # --- module level (X, Y), the five workloads at sizes that keep the fixtures small -------------------
    X, Y, lx, ly, w = make_inputs("readme")
    cases["mod_readme_f32"] = module_case(dist, X, Y, lx, ly, w.gamma, w.bandwidth, w.normalize)
    cases["mod_readme_f64"] = module_case(dist, X.double(), Y.double(), lx, ly, w.gamma, w.bandwidth, w.normalize)
    X, Y, lx, ly, w = make_inputs("medium", batch=4, N=96, M=80, d=64)
    cases["mod_medium_small_f32"] = module_case(dist, X, Y, lx, ly, w.gamma, w.bandwidth, w.normalize)
    cases["mod_medium_small_f64"] = module_case(dist, X.double(), Y.double(), lx, ly, w.gamma, w.bandwidth,
                                                w.normalize)
    X, Y, lx, ly, w = make_inputs("ragged", batch=8, N=64, M=48, d=8)
    cases["mod_ragged_small_f32"] = module_case(dist, X, Y, lx, ly, w.gamma, 8, w.normalize)
    cases["mod_ragged_small_f64"] = module_case(dist, X.double(), Y.double(), lx, ly, w.gamma, 8, w.normalize)
    X, Y, lx, ly, w = make_inputs("long", batch=2, N=300, M=280, d=16)
    cases["mod_long_small_f64"] = module_case(dist, X.double(), Y.double(), lx, ly, w.gamma, 24, w.normalize)
    X, Y, lx, ly, w = make_inputs("largebatch", batch=64, N=64, M=64, d=4)
    cases["mod_largebatch_small_f64"] = module_case(dist, X, Y, lx, ly, w.gamma, w.bandwidth, w.normalize)

    for name, arrays in cases.items():
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)
    total = sum(os.path.getsize(os.path.join(HERE, n + ".npz")) for n in cases)
    print(f"wrote {len(cases)} fixtures, {total / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
