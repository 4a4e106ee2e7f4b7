"""CPU: host logic of the library — the band rule as row intervals, the C ABI (exports, argument
checks that return before any launch), the op layer's validation (the reference's messages), the
FakeTensor kernels, the module's errors, and the seeded workloads. No kernel runs here."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT
from oracle import oracle as O
import torchsoftdtw_b200 as T
from torchsoftdtw_b200 import _ext, workloads


@pytest.fixture(scope="module")
def lib():
    return _ext.capi()


def header_functions():
    text = open(os.path.join(ROOT, "include", "sdtw_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sdtw_[a-z0-9_]+)\s*\(", text)))


def test_every_header_function_is_exported(lib):
    names = header_functions()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/sdtw_b200.h but not exported"
        assert name in _ext.SIGNATURES, f"{name} has no ctypes signature"


def test_debug_bounds_library_exports_the_same_functions():
    dbg = _ext.debug_capi()
    for name in header_functions():
        assert hasattr(dbg, name), f"{name} missing from the debug-bounds build"


def test_ops_library_links_kernel_library():
    import subprocess

    out = subprocess.run(["ldd", _ext.library_paths()[1]], capture_output=True, text=True).stdout
    assert "libsdtw_b200.so" in out


def _range(lib, i, nx, ny, bw):
    lo, hi = ctypes.c_int64(), ctypes.c_int64()
    lib.sdtw_band_row_range(i, nx, ny, bw, ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def test_band_row_range_matches_reference_predicate_exhaustive(lib):
    for nx in range(1, 13):
        for ny in range(1, 13):
            for bw in (-1, 0, 1, 2, 3, 5, 8, 100):
                for i in range(nx):
                    lo, hi = _range(lib, i, nx, ny, bw)
                    cols = [j for j in range(ny) if O.in_band(i, j, nx, ny, bw)]
                    assert cols, (nx, ny, bw, i)
                    assert (lo, hi) == (cols[0], cols[-1]), (nx, ny, bw, i)
                    assert cols == list(range(lo, hi + 1))  # the in-band set of a row is an interval


def test_band_row_range_random_large(lib):
    rng = np.random.default_rng(5)
    for _ in range(200):
        nx, ny = (int(v) for v in rng.integers(1, 3000, size=2))
        bw = int(rng.choice([-1, 0, 1, 7, 32, 256]))
        i = int(rng.integers(0, nx))
        lo, hi = _range(lib, i, nx, ny, bw)
        assert 0 <= lo <= hi < ny
        assert O.in_band(i, lo, nx, ny, bw) and O.in_band(i, hi, nx, ny, bw)
        assert lo == 0 or not O.in_band(i, lo - 1, nx, ny, bw)
        assert hi == ny - 1 or not O.in_band(i, hi + 1, nx, ny, bw)


def test_pair_cells_matches_oracle_count(lib):
    rng = np.random.default_rng(6)
    for _ in range(60):
        nx, ny = (int(v) for v in rng.integers(0, 90, size=2))
        bw = int(rng.choice([-1, 0, 1, 4, 16]))
        assert lib.sdtw_pair_cells(nx, ny, bw) == O.count_cells([nx], [ny], bw)


def test_status_strings(lib):
    assert lib.sdtw_status_string(0) == b"ok"
    for code in (-1, -2, -3, -4):
        assert len(lib.sdtw_status_string(code)) > 5


def test_c_abi_rejects_bad_arguments_before_launching(lib):
    null = None
    ws = ctypes.create_string_buffer(4096)
    # bad dtype, negative sizes, gamma <= 0, missing workspace: all return before touching the device
    assert lib.sdtw_forward(7, null, 1, 1, 1, null, null, 0, 1.0, -1, null, null, null, 0, null, null) == -2
    assert lib.sdtw_forward(0, null, -1, 1, 1, null, null, 0, 1.0, -1, null, null, null, 0, null, null) == -1
    assert lib.sdtw_forward(0, null, 1, 1, 1, null, null, 0, 0.0, -1, null, null, null, 0, null, null) == -1
    assert lib.sdtw_forward(0, null, 1, 1, 1, null, null, 0, float("nan"), -1, null, null, null, 0, null, null) == -1
    p = ctypes.cast(ws, ctypes.c_void_p)
    assert lib.sdtw_forward(0, p, 1, 4, 4, p, p, 0, 1.0, -1, p, p, null, 0, p, null) == -3
    assert lib.sdtw_backward(0, null, p, 1, 4, 4, p, p, 0, 1.0, -1, p, p, 1, p, null) == -3
    assert lib.sdtw_backward(1, null, null, 2, 4, 4, null, null, 0, -1.0, -1, null, null, 0, null, null) == -1
    assert lib.sdtw_pairwise_l2(3, null, null, 1, 1, 1, 1, null, null, null) == -2
    assert lib.sdtw_grad_l2(0, null, null, null, null, null, null, -2, 1, 1, 1, null, null, null) == -1
    # empty batch: nothing to do
    assert lib.sdtw_forward(0, null, 0, 4, 4, null, null, 0, 1.0, -1, null, null, null, 0, null, null) == 0
    # L1 / cosine entry points: unknown kind, eps <= 0, negative sizes, bad dtype, missing operands
    assert lib.sdtw_pairwise_dist(0, 3, p, p, 1, 4, 4, 2, 1e-8, p, null) == -1
    assert lib.sdtw_pairwise_dist(0, 2, p, p, 1, 4, 4, 2, 0.0, p, null) == -1
    assert lib.sdtw_pairwise_dist(0, 1, p, p, 1, -4, 4, 2, 1e-8, p, null) == -1
    assert lib.sdtw_pairwise_dist(5, 1, p, p, 1, 4, 4, 2, 1e-8, p, null) == -2
    assert lib.sdtw_pairwise_dist(0, 1, p, p, 1, 4, 4, 2, 1e-8, null, null) == -1  # no D
    assert lib.sdtw_pairwise_dist(0, 1, null, null, 0, 4, 4, 2, 1e-8, null, null) == 0  # empty batch
    assert lib.sdtw_grad_dist(0, 2, p, p, null, p, p, 1, 4, 4, 2, 1e-8, null, p, null, null) == -1  # cosine needs D
    assert lib.sdtw_grad_dist(0, 1, p, p, null, p, null, 1, 4, 4, 2, 1e-8, null, p, null, null) == -1  # no g
    assert lib.sdtw_grad_dist(0, 1, p, p, null, p, p, 1, 4, 4, 2, 1e-8, null, null, null, null) == 0  # no outputs
    assert lib.sdtw_grad_dist_workspace_bytes(256, 512, 0) >= 256 * 512 * 4
    assert lib.sdtw_grad_dist_workspace_bytes(256, 512, 1) >= 256 * 512 * 8


def test_fused_cost_forward_arguments(lib):
    """The fused cost forward's helpers and argument checks (no device needed: nothing is launched)."""
    null = None
    assert lib.sdtw_clamp_mask_words(256, 512, 512) == 256 * 512 * 16
    assert lib.sdtw_clamp_mask_words(2, 3, 33) == 2 * 3 * 2
    assert lib.sdtw_clamp_mask_words(-1, 3, 3) == 0
    # d must be a positive multiple of 16, and without a device no shape is accepted
    assert lib.sdtw_forward_l2_fused_ok(256, 512, 512, 8) == 0
    assert lib.sdtw_forward_l2_fused_ok(256, 512, 512, 0) == 0
    assert lib.sdtw_forward_l2_tiles(null, null, 1, 4, 4, 16, null, null, 0, 0.0, -1, null, null, null, null, null, 0,
                                     null, null) == -1  # gamma
    assert lib.sdtw_forward_l2_tiles(null, null, 0, 4, 4, 16, null, null, 0, 1.0, -1, null, null, null, null, null, 0,
                                     null, null) == 0  # empty batch
    assert lib.sdtw_apply_clamp_mask(null, null, null, -1, 4, 4, null) == -1
    assert lib.sdtw_apply_clamp_mask(null, null, null, 0, 4, 4, null) == 0
    assert lib.sdtw_apply_clamp_mask(null, null, null, 2, 4, 4, null) == -1  # missing buffers


def test_band_cost_and_gradient_arguments(lib):
    """The band-restricted cost and gradient: workspace size and argument checks (nothing is launched)."""
    null = None
    # 16 bytes of count, then one int per 128 x 128 tile
    assert lib.sdtw_pairwise_l2_band_workspace_bytes(16, 4096, 4096) == 16 + 4 * 16 * 32 * 32
    assert lib.sdtw_pairwise_l2_band_workspace_bytes(3, 129, 1) == 16 + 4 * 3 * 2 * 1
    assert lib.sdtw_pairwise_l2_band_workspace_bytes(-1, 4, 4) == 0
    buf = ctypes.c_void_p(4096)  # never dereferenced: every call below returns before any device work
    assert lib.sdtw_pairwise_l2_band(2, null, null, 1, 4, 4, 4, buf, buf, 0, 3, buf, null, buf, 64, null) == -2  # dtype
    assert lib.sdtw_pairwise_l2_band(0, null, null, 0, 4, 4, 4, null, null, 0, 3, null, null, null, 0, null) == 0
    assert lib.sdtw_pairwise_l2_band(0, buf, buf, 1, 4, 4, 4, null, buf, 0, 3, buf, null, buf, 64, null) == -1
    assert lib.sdtw_pairwise_l2_band(0, buf, buf, 1, 4, 4, 4, buf, buf, 0, 3, buf, null, buf, 8, null) == -3
    assert lib.sdtw_pairwise_l2_band(0, buf, buf, 1, 4, 4, 4, buf, buf, 0, 3, buf, null,
                                     ctypes.c_void_p(4100), 64, null) == -3  # workspace not 16-byte aligned
    assert lib.sdtw_grad_l2_band(0, buf, buf, buf, buf, buf, null, 1, 4, 4, 4, null, buf, 0, 3, buf, null,
                                 null) == -1


def test_fused_cost_policy_is_opt_in(monkeypatch):
    import torch

    from torchsoftdtw_b200 import _ext

    monkeypatch.delenv(_ext.FUSED_COST_ENV, raising=False)
    assert not _ext.l2_fused(256, 512, 512, 64, torch.float32, "cuda")
    monkeypatch.setenv(_ext.FUSED_COST_ENV, "1")
    assert not _ext.l2_fused(256, 512, 512, 64, torch.float64, "cuda")  # fp32 only
    assert not _ext.l2_fused(256, 512, 512, 64, torch.float32, "cpu")


def test_workspace_sizes(lib):
    f = lib.sdtw_forward_workspace_bytes(256, 512, 512, 0)
    b = lib.sdtw_backward_workspace_bytes(256, 512, 512, 0)
    assert f >= 256 * 16 * 512 * 4 and b >= 256 * 16 * 512 * 4  # one boundary row per strip
    assert lib.sdtw_backward_workspace_bytes(256, 512, 512, 1) > b


# ---- op layer on CPU tensors: the reference's TestInputValidation (test_robustness.py:139-184) ----

def test_validation_D_must_be_3d():
    with pytest.raises(RuntimeError, match="3D"):
        torch.ops.torchsoftdtw.forward(torch.rand(5, 5), torch.tensor([5]), torch.tensor([5]), 1.0, -1)


def test_validation_lengths_must_be_1d():
    with pytest.raises(RuntimeError, match="1D"):
        torch.ops.torchsoftdtw.forward(torch.rand(1, 5, 5), torch.tensor([[5]]), torch.tensor([5]), 1.0, -1)


def test_validation_batch_mismatch():
    with pytest.raises(RuntimeError, match="[Bb]atch"):
        torch.ops.torchsoftdtw.forward(torch.rand(2, 5, 5), torch.tensor([5, 5, 5]), torch.tensor([5, 5]), 1.0, -1)


def test_validation_gamma_must_be_positive():
    for g in (0.0, -1.0):
        with pytest.raises(RuntimeError, match="gamma"):
            torch.ops.torchsoftdtw.forward(torch.rand(1, 5, 5), torch.tensor([5]), torch.tensor([5]), g, -1)


def test_validation_D_must_be_float():
    with pytest.raises(RuntimeError, match="float"):
        torch.ops.torchsoftdtw.forward(torch.randint(0, 10, (1, 5, 5)), torch.tensor([5]), torch.tensor([5]), 1.0, -1)


def test_validation_lengths_must_be_int():
    with pytest.raises(RuntimeError, match="int"):
        torch.ops.torchsoftdtw.forward(torch.rand(1, 5, 5), torch.tensor([5.0]), torch.tensor([5]), 1.0, -1)


def test_backward_validation():
    with pytest.raises(RuntimeError, match="3D"):
        torch.ops.torchsoftdtw.backward(torch.rand(5, 5), torch.rand(1, 7, 7), torch.tensor([5]),
                                        torch.tensor([5]), 1.0, -1)


def test_cpu_tensors_are_rejected_without_fallback():
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        T.soft_dtw(torch.rand(2, 5, 7, dtype=torch.float64))
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        T.SoftDTW()(torch.randn(2, 5, 3), torch.randn(2, 6, 3))


def test_unknown_distance_raises():
    with pytest.raises(ValueError, match="Unknown distance"):
        T.SoftDTW(distance="manhattan")


def test_fake_tensor_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode() as mode:
        D = mode.from_tensor(torch.rand(2, 5, 7))
        lx = mode.from_tensor(torch.tensor([5, 5]))
        ly = mode.from_tensor(torch.tensor([7, 7]))
        costs, R = torch.ops.torchsoftdtw.forward(D, lx, ly, 1.0, -1)
        assert costs.shape == (2,) and R.shape == (2, 7, 9)
        E = torch.ops.torchsoftdtw.backward(D, mode.from_tensor(torch.rand(2, 7, 9)), lx, ly, 1.0, -1)
        assert E.shape == (2, 5, 7)
        Dh = mode.from_tensor(torch.rand(2, 5, 7, dtype=torch.float16))
        c16, R16 = torch.ops.torchsoftdtw.forward(Dh, lx, ly, 1.0, -1)
        assert c16.dtype == torch.float32 and R16.dtype == torch.float32
        assert torch.ops.torchsoftdtw.backward(Dh, R16, lx, ly, 1.0, -1).dtype == torch.float16
        X = mode.from_tensor(torch.rand(2, 5, 3))
        Y = mode.from_tensor(torch.rand(2, 7, 3))
        c, R, Dm, fl = torch.ops.torchsoftdtw_b200.l2_forward(X, Y, lx, ly, 1.0, -1)
        assert c.shape == (2,) and R.shape == (2, 7, 9) and Dm.shape == (2, 5, 7) and fl.dtype == torch.int32


def test_drop_in_import_name():
    import torchsoftdtw
    from torchsoftdtw.distances import pairwise_l2_squared
    from torchsoftdtw.softdtw import soft_dtw

    assert torchsoftdtw.SoftDTW is T.SoftDTW
    assert soft_dtw is T.soft_dtw and pairwise_l2_squared is T.pairwise_l2_squared


def test_workloads_are_seeded_and_shaped():
    X, Y, lx, ly, w = workloads.make_inputs("readme")
    assert X.shape == (8, 50, 16) and Y.shape == (8, 40, 16) and X.dtype == torch.float32
    X2, _, _, _, _ = workloads.make_inputs("readme")
    assert torch.equal(X, X2)
    X, Y, lx, ly, w = workloads.make_inputs("ragged", batch=64)
    assert X.shape == (64, 256, 32) and int(lx.min()) >= 64 and int(ly.max()) <= 192
    assert workloads.count_cells(lx, ly, w.bandwidth) == O.count_cells(lx.numpy(), ly.numpy(), w.bandwidth)
    X, Y, lx, ly, w = workloads.make_inputs("largebatch", batch=4)
    assert X.dtype == torch.float64 and float(X.abs().max()) <= 1.0


def test_headline_cell_count():
    _, _, lx, ly, w = workloads.make_inputs("medium", batch=2, d=1)
    assert workloads.count_cells(lx, ly, w.bandwidth) == 2 * 512 * 512


def test_benchmark_sweep_batches_and_table():
    """The sweep's batches follow the spread rules (lengths in [ceil-ish fraction * L, L], frames past a
    sample's length zeroed) and the table has one row per measurement."""
    import torch

    from torchsoftdtw_b200 import benchmark as bm

    for spread, lo in bm.SPREADS.items():
        X, Y, lx, ly = bm.make_batch(16, 40, 3, spread, torch.device("cpu"), seed=1)
        assert X.shape == (16, 40, 3) and Y.shape == (16, 40, 3)
        first = max(1, round(lo * 40))
        for t, lens in ((X, lx), (Y, ly)):
            assert int(lens.min()) >= first and int(lens.max()) <= 40
            for b in range(16):
                assert torch.count_nonzero(t[b, int(lens[b]):]) == 0
    rows = [{"B": 2, "L": 8, "D": 1, "spread": "none", "cells": 128.0, "fwd_ms": 0.5, "fwdbwd_ms": 1.0}]
    text = bm.table(rows, "dev")
    assert text.count("\n| 2 | 8 | 1 | none |") == 1 and "2.560e+05" in text
    rows[0]["unfused_fwdbwd_ms"] = 3.0
    text = bm.table(rows, "dev", "l1", 0.1)
    assert "distance = l1" in text and "gamma = 0.1" in text and text.rstrip().endswith("| 3.000 |")
