"""GPU parity of the fused squared-L2 forward (sdtw_forward_l2_tiles: the cost matrix computed tile by tile
inside the pair-resident forward wavefront and never stored), opt-in on the module path with
TORCHSOFTDTW_B200_FUSED_COST=1.

Checked against the stored-D pair (sdtw_pairwise_l2 + sdtw_forward_tiles, itself oracle-checked) through
the C ABI, and against the oracle's module restatement through SoftDTW. Tolerances: fp32 costs rtol 1e-5 /
atol 1e-6 (the products are 3xTF32 in both cost paths, summed in different orders); fp32 gradients by the
module contract of tests/test_gpu_module.py."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
import torchsoftdtw_b200 as T
from torchsoftdtw_b200 import _ext

from test_gpu_module import grad_contract, run_module

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def fused_vs_stored(dev, B, N, M, d, bw=-1, ragged=False, same=False, seed=0, gamma=0.1):
    """Costs and E (from sdtw_backward_tiles on each forward's R tiles) of the fused forward and of the
    stored-D pair on the same seeded inputs; plus the clamp records of both."""
    lib = _ext.capi()
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(B, N, d, generator=g)
    Y = X[:, :M].clone() if same else torch.randn(B, M, d, generator=g)
    if ragged:
        lx = torch.randint(max(1, N // 2), N + 1, (B,), generator=g)
        ly = torch.randint(max(1, M // 2), M + 1, (B,), generator=g)
    else:
        lx, ly = torch.full((B,), N), torch.full((B,), M)
    X, Y, lx, ly = X.to(dev), Y.to(dev), lx.to(dev), ly.to(dev)
    assert lib.sdtw_forward_l2_fused_ok(B, N, M, d) == 1
    sp = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    S, NBt = (N + 31) // 32, (M + 31) // 32 + 1
    D = torch.empty(B, N, M, device=dev)
    flags = torch.zeros(B, device=dev, dtype=torch.int32)
    err = torch.zeros(1, device=dev, dtype=torch.int32)
    ws = torch.empty(max(lib.sdtw_forward_workspace_bytes(B, N, M, 0), lib.sdtw_backward_workspace_bytes(B, N, M, 0)),
                     device=dev, dtype=torch.uint8)
    out = {}
    for fused in (False, True):
        Rt = torch.empty(B, S, NBt, 32, 32, device=dev)
        c = torch.empty(B, device=dev)
        E = torch.empty(B, N, M, device=dev)
        if fused:
            mask = torch.empty(lib.sdtw_clamp_mask_words(B, N, M), device=dev, dtype=torch.int32)
            cfl = torch.empty(B, device=dev, dtype=torch.int32)
            st = lib.sdtw_forward_l2_tiles(_p(X), _p(Y), B, N, M, d, _p(lx), _p(ly), 0, gamma, bw, _p(Rt), _p(c),
                                           _p(mask), _p(cfl), _p(ws), ws.numel(), _p(err), sp)
        else:
            assert lib.sdtw_pairwise_l2(0, _p(X), _p(Y), B, N, M, d, _p(D), _p(flags), sp) == 0
            st = lib.sdtw_forward_tiles(0, _p(D), B, N, M, _p(lx), _p(ly), 0, gamma, bw, _p(Rt), _p(c), _p(ws),
                                        ws.numel(), _p(err), sp)
        assert st == 0
        assert lib.sdtw_backward_tiles(0, _p(Rt), B, N, M, _p(lx), _p(ly), 0, gamma, bw, _p(E), _p(ws), ws.numel(),
                                       _p(err), sp) == 0
        torch.cuda.synchronize()
        assert lib.sdtw_read_error_word(_p(err), sp) == 0
        out["fused" if fused else "stored"] = (c.cpu(), E.cpu())
        if fused:
            out["mask"], out["cflags"] = mask.view(B, N, (M + 31) // 32).cpu(), cfl.cpu()
    out["D"], out["flags"] = D.cpu(), flags.cpu()
    out["lx"], out["ly"] = lx.cpu(), ly.cpu()
    return out


@pytest.mark.parametrize("shape", [dict(B=256, N=512, M=512, d=64), dict(B=64, N=300, M=280, d=32, ragged=True),
                                   dict(B=40, N=256, M=384, d=48, bw=40, ragged=True),
                                   dict(B=148, N=192, M=200, d=16), dict(B=20, N=500, M=130, d=128, ragged=True)],
                         ids=["medium", "ragged_d32", "band_d48", "d16", "d128"])
def test_fused_forward_equals_stored_cost_path(cuda, shape):
    r = fused_vs_stored(cuda, **shape)
    (cs, Es), (cf, Ef) = r["stored"], r["fused"]
    torch.testing.assert_close(cf, cs, rtol=1e-5, atol=1e-6)
    # E from the two forwards' R tiles. At gamma = 0.1, R ~ 1e4 and one ulp of R is ~1e-2 gamma, so two fp32
    # forwards whose D differ in the last bits give softmin weights that differ by up to the fp32 path's own
    # error against fp64 (0.068 on the medium workload; the reference's fp32 backward: 0.67). Bound: 0.05
    # absolute anywhere, and all but 1e-3 of the cells within 5e-5 (measured: at most 1.3e-4).
    diff = (Ef - Es).abs()
    assert float(diff.max()) <= 0.05, float(diff.max())
    assert float((diff > 5e-5).float().mean()) <= 1e-3
    assert int(r["cflags"].ne(0).sum()) == 0 and int(r["mask"].ne(0).sum()) == 0  # N(0,1) data: no clamp


def test_fused_clamp_mask_marks_negative_cells(cuda):
    # Identical sequences: |x|^2 + |y|^2 - 2 x.y rounds to either side of 0 on the diagonal. Every bit of the
    # fused forward's clamp mask is a diagonal cell inside the lengths, and its flag is set with it.
    B, N, d = 32, 192, 64
    r = fused_vs_stored(cuda, B, N, N, d, same=True, seed=4)
    mask, cfl = r["mask"], r["cflags"]
    bits = np.unpackbits(mask.numpy().view(np.uint8), bitorder="little").reshape(B, N, -1)[:, :, :N]
    ii, jj = np.nonzero(bits.any(axis=0))
    assert np.all(ii == jj), "a clamped cell off the diagonal"
    assert np.array_equal(bits.reshape(B, -1).any(axis=1), cfl.numpy() != 0)
    # The exact cost is 0 (every diagonal D is 0); both fp32 cost paths give the sum of the diagonal's
    # rounding residues, each a few ulps of |x|^2 + |y|^2 ~ 128 (ulp 2^-16): at most N * 8 ulps.
    (cs, _), (cf, _) = r["stored"], r["fused"]
    bound = N * 8 * 2.0**-16
    assert float(cs.abs().max()) <= bound and float(cf.abs().max()) <= bound, (cs.abs().max(), cf.abs().max())


@pytest.fixture
def fused_env(monkeypatch):
    monkeypatch.setenv(_ext.FUSED_COST_ENV, "1")
    yield


@pytest.mark.parametrize("ragged", [False, True])
def test_module_fused_cost_vs_oracle(cuda, fused_env, ragged):
    g = torch.Generator().manual_seed(11)
    B, N, M, d = 24, 200, 176, 32
    X = torch.randn(B, N, d, generator=g)
    Y = torch.randn(B, M, d, generator=g)
    lx = torch.randint(N // 2, N + 1, (B,), generator=g) if ragged else torch.full((B,), N)
    ly = torch.randint(M // 2, M + 1, (B,), generator=g) if ragged else torch.full((B,), M)
    bw = 30 if ragged else -1
    assert _ext.l2_fused(B, N, M, d, torch.float32, cuda)
    c, gx, gy = run_module(X, Y, lx, ly, 0.5, bw, True, cuda)
    c64, _, _ = O.module_forward_backward(X.double().numpy(), Y.double().numpy(), lx.numpy(), ly.numpy(), 0.5, bw,
                                          True)
    np.testing.assert_allclose(c, c64, rtol=1e-5, atol=1e-6)
    grad_contract(gx, X.numpy(), Y.numpy(), lx.numpy(), ly.numpy(), 0.5, bw, True, "x")
    grad_contract(gy, X.numpy(), Y.numpy(), lx.numpy(), ly.numpy(), 0.5, bw, True, "y")


def test_module_fused_cost_clamped_pairs(cuda, fused_env):
    # Pairs with clamped cells: the clamp mask zeroes their gradient there, as the stored D's sign does.
    torch.manual_seed(5)
    B, N, d = 16, 192, 64
    X = torch.randn(B, N, d)
    Y = X.clone()
    Y[::2] += 0.05 * torch.randn(B // 2, N, d)
    lx, ly = torch.full((B,), N), torch.full((B,), N)
    assert _ext.l2_fused(B, N, N, d, torch.float32, cuda)
    c, gx, gy = run_module(X, Y, lx, ly, 0.1, -1, False, cuda)
    assert np.isfinite(c).all() and np.isfinite(gx).all() and np.isfinite(gy).all()
    grad_contract(gx, X.numpy(), Y.numpy(), lx.numpy(), ly.numpy(), 0.1, -1, False, "x")


def test_module_fused_cost_off_by_default(cuda, monkeypatch):
    monkeypatch.delenv(_ext.FUSED_COST_ENV, raising=False)
    assert not _ext.l2_fused(256, 512, 512, 64, torch.float32, cuda)
    X = torch.randn(256, 512, 64, device=cuda)
    _, _, D, _ = torch.ops.torchsoftdtw_b200.l2_forward(X, X, torch.full((256,), 512, device=cuda),
                                                        torch.full((256,), 512, device=cuda), 0.1, -1)
    assert D.dtype == torch.float32 and D.shape == (256, 512, 512)
