"""GPU: the L1 and cosine cost-matrix and gradient kernels (C ABI ``sdtw_pairwise_dist`` / ``sdtw_grad_dist``)
and the module path built on them.

* cost matrices against fp64 numpy restatements of the reference's expressions
  (``src/torchsoftdtw/distances.py:21-50``), fp32 and fp64, tiles and feature chunks cut at any size,
  zero-norm rows for cosine (norm floored at eps);
* gradients against fp64 torch autograd of the same expressions, weighted by a per-pair g and a cell
  weight E (the contraction ``sum_b g[b] sum_ij E[b,i,j] dD[b,i,j]`` the module's backward needs);
* the module (``SoftDTW(distance="l1"|"cosine")``) against the unfused composition expression -> soft_dtw,
  and gradcheck in fp64.
"""

import ctypes

import numpy as np
import pytest
import torch

import torchsoftdtw_b200 as T
from torchsoftdtw_b200 import _ext

pytestmark = pytest.mark.gpu

KIND = {"l1": 1, "cosine": 2}
EPS = 1e-8
p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dist(kind, X, Y, eps=EPS):
    lib = _ext.capi()
    B, N, d = X.shape
    M = Y.shape[1]
    D = torch.empty(B, N, M, device=X.device, dtype=X.dtype)
    st = lib.sdtw_pairwise_dist(1 if X.dtype == torch.float64 else 0, KIND[kind], p(X), p(Y), B, N, M, d, eps, p(D),
                                stream())
    assert st == 0, lib.sdtw_status_string(st)
    torch.cuda.synchronize()
    return D


def grad(kind, X, Y, D, E, g, need_x=True, need_y=True, eps=EPS, workspace=True):
    lib = _ext.capi()
    B, N, d = X.shape
    M = Y.shape[1]
    dt = 1 if X.dtype == torch.float64 else 0
    gX = torch.empty_like(X) if need_x else None
    gY = torch.empty_like(Y) if need_y else None
    ws = torch.empty(lib.sdtw_grad_dist_workspace_bytes(B, M, dt), dtype=torch.uint8, device=X.device) if workspace \
        else None
    st = lib.sdtw_grad_dist(dt, KIND[kind], p(X), p(Y), p(D), p(E), p(g), B, N, M, d, eps, p(ws), p(gX), p(gY),
                            stream())
    assert st == 0, lib.sdtw_status_string(st)
    torch.cuda.synchronize()
    return gX, gY


def np_l1(X, Y):
    return np.abs(X[:, :, None, :] - Y[:, None, :, :]).sum(-1)


def np_cosine(X, Y, eps=EPS):
    nx = np.maximum(np.linalg.norm(X, axis=-1), eps)
    ny = np.maximum(np.linalg.norm(Y, axis=-1), eps)
    return 1.0 - np.einsum("bik,bjk->bij", X, Y) / (nx[:, :, None] * ny[:, None, :])


def inputs(B, N, M, d, seed, dtype, zero_rows=False):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(B, N, d, generator=g, dtype=torch.float64)
    Y = torch.randn(B, M, d, generator=g, dtype=torch.float64)
    if zero_rows:
        X[:, ::5] = 0.0
        Y[:, 1::7] = 0.0
    return X, Y


SHAPES = [(1, 1, 1, 1), (2, 7, 5, 3), (3, 64, 64, 16), (2, 65, 130, 17), (1, 200, 96, 40), (2, 33, 300, 129),
          (2, 130, 260, 64), (1, 300, 132, 128), (3, 129, 64, 12), (1, 64, 520, 200)]

# Cosine in fp32 runs the tcgen05 kernels where the shape allows (auto); "cuda_cores" forces the
# CUDA-core kernels.
DISTANCE_PATHS = {"auto": 0, "cuda_cores": 2}


@pytest.fixture(params=list(DISTANCE_PATHS))
def distance_path(request):
    lib = _ext.capi()
    lib.sdtw_debug_force_distance_path(DISTANCE_PATHS[request.param])
    yield request.param
    lib.sdtw_debug_force_distance_path(0)


@pytest.mark.parametrize("kind", ["l1", "cosine"])
@pytest.mark.parametrize("B,N,M,d", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_cost_matches_fp64(cuda, distance_path, kind, B, N, M, d, dtype):
    X, Y = inputs(B, N, M, d, 1000 + N + M + d, dtype, zero_rows=(kind == "cosine"))
    Xd, Yd = X.to(dtype), Y.to(dtype)
    D = dist(kind, Xd.to(cuda), Yd.to(cuda)).cpu().double().numpy()
    ref = (np_l1 if kind == "l1" else np_cosine)(Xd.double().numpy(), Yd.double().numpy())
    if dtype == torch.float64:
        np.testing.assert_allclose(D, ref, rtol=1e-12, atol=1e-12)
    elif kind == "l1":
        # fp32 sum of d terms |x - y|: relative error a few ulp times d
        np.testing.assert_allclose(D, ref, rtol=4e-7 * max(d, 4), atol=1e-6)
    else:
        np.testing.assert_allclose(D, ref, rtol=0, atol=2e-6)


@pytest.mark.parametrize("kind", ["l1", "cosine"])
@pytest.mark.parametrize("B,N,M,d", SHAPES[1:])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_grad_matches_autograd_fp64(cuda, distance_path, kind, B, N, M, d, dtype):
    X, Y = inputs(B, N, M, d, 2000 + N + M + d, dtype, zero_rows=(kind == "cosine"))
    gen = torch.Generator().manual_seed(7)
    E = torch.rand(B, N, M, generator=gen, dtype=torch.float64)
    E[:, :, -1:] = 0.0  # padded columns carry no weight
    g = torch.rand(B, generator=gen, dtype=torch.float64) + 0.5

    Xr = X.to(dtype).double().requires_grad_(True)
    Yr = Y.to(dtype).double().requires_grad_(True)
    Dr = (T.pairwise_l1 if kind == "l1" else T.pairwise_cosine)(Xr, Yr)
    (g[:, None, None] * E * Dr).sum().backward()

    Xc, Yc = X.to(dtype).to(cuda), Y.to(dtype).to(cuda)
    D = dist(kind, Xc, Yc)
    Ec, gc = E.to(dtype).to(cuda), g.to(dtype).to(cuda)
    gX, gY = grad(kind, Xc, Yc, D, Ec, gc)
    gX_nows, _ = grad(kind, Xc, Yc, D, Ec, gc, need_y=False, workspace=False)  # no workspace: CUDA cores
    tol = 1e-11 if dtype == torch.float64 else 2e-5
    for ours, ref, A in ((gX, Xr.grad, X), (gY, Yr.grad, Y), (gX_nows, Xr.grad, X)):
        ours = ours.cpu().double()
        # rows of zero norm (cosine) have gradients ~1/eps: check them and the others at their own scales
        live = A.norm(dim=-1) > 0
        for sel in (live, ~live):
            if sel.any():
                scale = ref[sel].abs().max().item() + 1e-30
                err = (ours[sel] - ref[sel]).abs().max().item() / scale
                assert err < tol, (kind, err)


@pytest.mark.parametrize("kind", ["l1", "cosine"])
@pytest.mark.parametrize("M,d", [(30, 9), (32, 16)])
def test_grad_selection(cuda, kind, M, d):
    X, Y = inputs(2, 40, M, d, 5, torch.float32)
    Xc, Yc = X.float().to(cuda), Y.float().to(cuda)
    D = dist(kind, Xc, Yc)
    E = torch.rand(2, 40, M, device=cuda)
    g = torch.ones(2, device=cuda)
    gx_both, gy_both = grad(kind, Xc, Yc, D, E, g)
    gx, none = grad(kind, Xc, Yc, D, E, g, need_y=False)
    assert none is None and torch.equal(gx, gx_both)
    none, gy = grad(kind, Xc, Yc, D, E, g, need_x=False)
    assert none is None and torch.equal(gy, gy_both)


def test_invalid_arguments_are_rejected(cuda):
    lib = _ext.capi()
    X = torch.zeros(1, 4, 3, device=cuda)
    D = torch.empty(1, 4, 4, device=cuda)
    assert lib.sdtw_pairwise_dist(0, 3, p(X), p(X), 1, 4, 4, 3, EPS, p(D), stream()) != 0  # unknown kind
    assert lib.sdtw_pairwise_dist(0, 2, p(X), p(X), 1, 4, 4, 3, 0.0, p(D), stream()) != 0  # eps <= 0
    assert lib.sdtw_pairwise_dist(0, 1, p(X), p(X), 1, 4, 4, -1, EPS, p(D), stream()) != 0  # negative d


@pytest.mark.parametrize("distance", ["l1", "cosine"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("M,d", [(37, 6), (36, 8)])  # (36, 8) takes the tensor-core cosine kernels in fp32
def test_module_matches_unfused_composition(cuda, distance, dtype, M, d):
    g = torch.Generator().manual_seed(41)
    X = torch.randn(4, 50, d, generator=g, dtype=dtype)
    Y = torch.randn(4, M, d, generator=g, dtype=dtype)
    lx = torch.tensor([50, 44, 20, 1])
    ly = torch.tensor([M, 30, M, 5])
    module = T.SoftDTW(gamma=0.3, normalize=True, bandwidth=12, distance=distance)

    X1 = X.to(cuda).requires_grad_(True)
    Y1 = Y.to(cuda).requires_grad_(True)
    c1 = module(X1, Y1, lx.to(cuda), ly.to(cuda))
    c1.sum().backward()

    X2 = X.to(cuda).requires_grad_(True)
    Y2 = Y.to(cuda).requires_grad_(True)
    expr = T.pairwise_l1 if distance == "l1" else T.pairwise_cosine
    c2 = T.soft_dtw(expr(X2, Y2), lx.to(cuda), ly.to(cuda), 0.3, 12)
    c2 = c2 / (lx.to(cuda) + ly.to(cuda) - 1).to(c2.dtype)
    c2.sum().backward()

    tol = dict(rtol=1e-10, atol=1e-10) if dtype == torch.float64 else dict(rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(c1, c2, **tol)
    torch.testing.assert_close(X1.grad, X2.grad, **tol)
    torch.testing.assert_close(Y1.grad, Y2.grad, **tol)


@pytest.mark.parametrize("distance", ["l1", "cosine"])
def test_module_gradcheck(cuda, distance):
    g = torch.Generator().manual_seed(43)
    X = torch.randn(2, 9, 4, generator=g, dtype=torch.float64).to(cuda).requires_grad_(True)
    Y = torch.randn(2, 7, 4, generator=g, dtype=torch.float64).to(cuda).requires_grad_(True)
    lx = torch.tensor([9, 6], device=cuda)
    ly = torch.tensor([7, 7], device=cuda)
    module = T.SoftDTW(gamma=0.5, distance=distance)
    assert torch.autograd.gradcheck(lambda a, b: module(a, b, lx, ly), (X, Y), eps=1e-6, atol=1e-6)


@pytest.mark.parametrize("kind", ["l1", "cosine"])
def test_batches_above_the_grid_limit(cuda, kind):
    """B = 65537 pairs: cost matrices and gradients of the chunked launches against fp64 autograd."""
    B, N, M, d = 65537, 5, 4, 8
    X, Y = inputs(B, N, M, d, 9, torch.float32)
    gen = torch.Generator().manual_seed(10)
    E = torch.rand(B, N, M, generator=gen, dtype=torch.float64)
    g = torch.rand(B, generator=gen, dtype=torch.float64)
    Xr = X.float().double().requires_grad_(True)
    Yr = Y.float().double().requires_grad_(True)
    Dr = (T.pairwise_l1 if kind == "l1" else T.pairwise_cosine)(Xr, Yr)
    (g[:, None, None] * E * Dr).sum().backward()
    Xc, Yc = X.float().to(cuda), Y.float().to(cuda)
    D = dist(kind, Xc, Yc)
    torch.testing.assert_close(D.double().cpu(), Dr.detach(), rtol=1e-5, atol=1e-5)
    gX, gY = grad(kind, Xc, Yc, D, E.float().to(cuda), g.float().to(cuda))
    torch.testing.assert_close(gX.double().cpu(), Xr.grad, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(gY.double().cpu(), Yr.grad, rtol=1e-4, atol=1e-4)
