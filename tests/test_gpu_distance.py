"""GPU: the cost-matrix and gradient kernels called through the C ABI, against fp64 numpy.

* fp32 cost matrix on every path (tcgen05 tensor cores, mma.sync, CUDA cores; both tensor-core paths in
  3xTF32): D within 2e-6 of the fp64 value relative to |x|^2 + |y|^2, the clamp recorded as -0.0,
  per-pair clamp flags consistent with the sign bits, tiles and feature chunks cut at any size;
* grad_X / grad_Y: against 2*g*(rowsum(G) X - G Y) in fp64 with G = E * mask, for masked and unmasked
  pairs, and for shapes that take the CUDA-core kernels.
"""

import ctypes

import numpy as np
import pytest
import torch

from torchsoftdtw_b200 import _ext

pytestmark = pytest.mark.gpu

p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def pairwise(X, Y, flags=True):
    lib = _ext.capi()
    B, N, d = X.shape
    M = Y.shape[1]
    D = torch.empty(B, N, M, device=X.device, dtype=X.dtype)
    fl = torch.full((B,), 7, device=X.device, dtype=torch.int32) if flags else None
    st = lib.sdtw_pairwise_l2(1 if X.dtype == torch.float64 else 0, p(X), p(Y), B, N, M, d, p(D), p(fl), stream())
    assert st == 0, lib.sdtw_status_string(st)
    torch.cuda.synchronize()
    return D, fl


def grad(X, Y, D, E, g, flags, need_x=True, need_y=True):
    lib = _ext.capi()
    B, N, d = X.shape
    M = Y.shape[1]
    gX = torch.empty_like(X) if need_x else None
    gY = torch.empty_like(Y) if need_y else None
    st = lib.sdtw_grad_l2(1 if X.dtype == torch.float64 else 0, p(X), p(Y), p(D), p(E), p(g), p(flags), B, N, M, d,
                          p(gX), p(gY), stream())
    assert st == 0, lib.sdtw_status_string(st)
    torch.cuda.synchronize()
    return gX, gY


SHAPES = [(3, 130, 70, 64), (2, 64, 64, 4), (2, 33, 257, 16), (1, 300, 200, 128), (2, 5, 7, 8), (2, 128, 128, 12),
          (1, 17, 19, 3), (2, 130, 132, 64), (3, 64, 64, 36), (2, 257, 260, 8), (1, 129, 4, 4), (1, 40, 384, 100)]

# 0: chosen by shape (tcgen05 where d % 4 == 0 and M % 4 == 0, then the narrow kernels where d <= 16),
# 1: mma.sync kernels, 2: tiled CUDA-core kernels, 3: narrow CUDA-core kernels (d <= 16)
DISTANCE_PATHS = [0, 1, 2, 3]


@pytest.fixture(params=DISTANCE_PATHS)
def distance_path(request):
    lib = _ext.capi()
    lib.sdtw_debug_force_distance_path(request.param)
    yield request.param
    lib.sdtw_debug_force_distance_path(0)


@pytest.mark.parametrize("B,N,M,d", SHAPES)
def test_pairwise_fp32_accuracy_and_clamp_sign(cuda, distance_path, B, N, M, d):
    g = torch.Generator().manual_seed(N * M + d)
    X = torch.randn(B, N, d, generator=g)
    Y = torch.randn(B, M, d, generator=g)
    Y[0, : min(N, M) // 2] = X[0, : min(N, M) // 2]  # identical frames: values near 0, some clamped
    D, fl = pairwise(X.to(cuda), Y.to(cuda))
    Dn = D.cpu().numpy()
    Xd, Yd = X.double().numpy(), Y.double().numpy()
    x2, y2 = (Xd * Xd).sum(-1), (Yd * Yd).sum(-1)
    exact = x2[:, :, None] + y2[:, None, :] - 2 * np.matmul(Xd, np.swapaxes(Yd, 1, 2))
    scale = x2[:, :, None] + y2[:, None, :] + 1e-30
    assert np.max(np.abs(Dn - np.maximum(exact, 0)) / scale) < 2e-6
    neg = np.signbit(Dn)
    assert np.all(Dn[neg] == 0.0) and np.all(Dn >= 0)
    assert np.array_equal(fl.cpu().numpy() != 0, neg.reshape(B, -1).any(1))


def test_pairwise_fp64_matches_numpy(cuda, distance_path):
    g = torch.Generator().manual_seed(3)
    X = torch.rand(4, 40, 4, generator=g, dtype=torch.float64) * 2 - 1
    Y = torch.rand(4, 33, 4, generator=g, dtype=torch.float64) * 2 - 1
    D, _ = pairwise(X.to(cuda), Y.to(cuda))
    Xd, Yd = X.numpy(), Y.numpy()
    exact = (Xd * Xd).sum(-1)[:, :, None] + (Yd * Yd).sum(-1)[:, None, :] - 2 * np.matmul(Xd, np.swapaxes(Yd, 1, 2))
    np.testing.assert_allclose(D.cpu().numpy(), np.maximum(exact, 0), rtol=1e-13, atol=1e-13)


def reference_grads(X, Y, D, E, g):
    Xd, Yd = X.double().cpu().numpy(), Y.double().cpu().numpy()
    mask = ~np.signbit(D.cpu().numpy())
    G = g.double().cpu().numpy()[:, None, None] * E.double().cpu().numpy() * mask
    gx = 2 * (G.sum(2)[:, :, None] * Xd - np.matmul(G, Yd))
    gy = 2 * (G.sum(1)[:, :, None] * Yd - np.matmul(np.swapaxes(G, 1, 2), Xd))
    return gx, gy


@pytest.mark.parametrize("B,N,M,d", [(2, 130, 72, 64), (3, 64, 64, 4), (1, 257, 100, 128), (2, 40, 36, 12),
                                     (2, 9, 10, 3), (2, 128, 130, 16)])
@pytest.mark.parametrize("force_mask", [False, True])
def test_grad_matches_fp64(cuda, distance_path, B, N, M, d, force_mask):
    gen = torch.Generator().manual_seed(B + N + M + d)
    X = torch.randn(B, N, d, generator=gen)
    Y = torch.randn(B, M, d, generator=gen)
    E = torch.rand(B, N, M, generator=gen)
    D = torch.rand(B, N, M, generator=gen) + 0.1
    if force_mask:
        D[torch.rand(B, N, M, generator=gen) < 0.1] = -0.0
    gvec = torch.rand(B, generator=gen) + 0.5
    flags = torch.tensor([1 if force_mask else 0] * B, dtype=torch.int32)
    Xc, Yc, Dc, Ec, gc, fc = (t.to(cuda) for t in (X, Y, D, E, gvec, flags))
    gX, gY = grad(Xc, Yc, Dc, Ec, gc, fc)
    ex, ey = reference_grads(X, Y, D, E, gvec)
    scale_x = np.max(np.abs(ex)) + 1e-30
    scale_y = np.max(np.abs(ey)) + 1e-30
    assert np.max(np.abs(gX.cpu().numpy() - ex)) / scale_x < 2e-6
    assert np.max(np.abs(gY.cpu().numpy() - ey)) / scale_y < 2e-6
    # no flags at all: every pair is treated as possibly clamped
    gX2, _ = grad(Xc, Yc, Dc, Ec, gc, None, need_y=False)
    assert np.max(np.abs(gX2.cpu().numpy() - ex)) / scale_x < 2e-6


@pytest.mark.parametrize("B,N,M,d", [(8, 512, 512, 64), (3, 300, 200, 32), (2, 37, 260, 128), (2, 64, 4, 16)])
@pytest.mark.parametrize("masked", [False, True])
def test_grad_y_tensor_cores(cuda, B, N, M, d, masked):
    """grad_Y on the tcgen05 kernel (E read transposed: output rows are E's columns, K runs over its rows, in
    chunks whose last one is ragged) against the fp64 contraction, and against the CUDA-core kernel."""
    gen = torch.Generator().manual_seed(B * N + M + d)
    X = torch.randn(B, N, d, generator=gen)
    Y = torch.randn(B, M, d, generator=gen)
    E = torch.rand(B, N, M, generator=gen)
    D = torch.rand(B, N, M, generator=gen) + 0.1
    if masked:
        D[torch.rand(B, N, M, generator=gen) < 0.1] = -0.0
    gvec = torch.rand(B, generator=gen) + 0.5
    flags = torch.tensor([1 if masked else 0] * B, dtype=torch.int32)
    Xc, Yc, Dc, Ec, gc, fc = (t.to(cuda) for t in (X, Y, D, E, gvec, flags))
    _, gY = grad(Xc, Yc, Dc, Ec, gc, fc, need_x=False)
    _, ey = reference_grads(X, Y, D, E, gvec)
    scale = np.max(np.abs(ey)) + 1e-30
    assert np.max(np.abs(gY.cpu().numpy() - ey)) / scale < 2e-6
    lib = _ext.capi()
    try:
        lib.sdtw_debug_force_distance_path(2)
        _, gY_cc = grad(Xc, Yc, Dc, Ec, gc, fc, need_x=False)
    finally:
        lib.sdtw_debug_force_distance_path(0)
    assert float((gY - gY_cc).abs().max()) / scale < 4e-6


def test_tensor_core_paths_agree(cuda):
    """tcgen05 and mma.sync cost matrices of the headline shape agree to fp32 rounding."""
    lib = _ext.capi()
    g = torch.Generator().manual_seed(11)
    X = torch.randn(4, 512, 64, generator=g).to(cuda)
    Y = torch.randn(4, 512, 64, generator=g).to(cuda)
    try:
        D_tc, f_tc = pairwise(X, Y)
        lib.sdtw_debug_force_distance_path(1)
        D_mma, f_mma = pairwise(X, Y)
    finally:
        lib.sdtw_debug_force_distance_path(0)
    scale = (X * X).sum(-1)[:, :, None] + (Y * Y).sum(-1)[:, None, :]
    assert float(((D_tc - D_mma).abs() / scale).max()) < 2e-6
    assert torch.equal(f_tc, f_mma)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_batches_above_the_grid_limit(cuda, dtype):
    """B = 65537 pairs (more than one launch's grid.z): the entry points run the batch in chunks; every
    pair's cost matrix and gradient match those computed pair-chunk by pair-chunk in fp64."""
    B, N, M, d = 65537, 5, 3, 4
    g0 = torch.Generator().manual_seed(3)
    X = torch.randn(B, N, d, generator=g0, dtype=torch.float64)
    Y = torch.randn(B, M, d, generator=g0, dtype=torch.float64)
    E = torch.rand(B, N, M, generator=g0, dtype=torch.float64)
    gg = torch.rand(B, generator=g0, dtype=torch.float64)
    Xc, Yc = X.to(dtype).to(cuda), Y.to(dtype).to(cuda)
    D, fl = pairwise(Xc, Yc)
    ref = (X.pow(2).sum(-1)[:, :, None] + Y.pow(2).sum(-1)[:, None, :] - 2 * X @ Y.transpose(1, 2)).clamp_min(0)
    tol = 1e-10 if dtype == torch.float64 else 1e-4
    torch.testing.assert_close(D.double().cpu(), ref, rtol=tol, atol=tol)
    gX, gY = grad(Xc, Yc, D, E.to(dtype).to(cuda), gg.to(dtype).to(cuda), fl)
    G = E * gg[:, None, None] * (ref > 0)
    gx_ref = 2 * (G.sum(2, keepdim=True) * X - G @ Y)
    gy_ref = 2 * (G.sum(1).unsqueeze(-1) * Y - G.transpose(1, 2) @ X)
    torch.testing.assert_close(gX.double().cpu(), gx_ref, rtol=tol, atol=tol)
    torch.testing.assert_close(gY.double().cpu(), gy_ref, rtol=tol, atol=tol)
