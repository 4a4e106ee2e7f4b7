"""ORACLE — test infrastructure only; the product package never imports this module.

ctypes front end for two CPU checkers:

* ``liboracle_softdtw.so`` — the plain-C restatement of the reference CPU operator
  (``src/torchsoftdtw/csrc/softdtw.cpp:97-285``, ``band.h:23-38``), built by ``make -C oracle``;
* ``_ref/libsoftdtw_ref_cpu.so`` — the reference's own CPU operator compiled from its source file
  (``make -C oracle ref``; only possible where the reference sources exist). It registers the ops
  ``torch.ops.torchsoftdtw_ref.forward/backward`` with the reference's schemas;
* ``_ref/libsoftdtw_ref_cuda.so`` — the reference's CUDA operator (``csrc/cuda/softdtw.cu``) compiled from
  its sources for sm_100 (``make -C oracle ref-cuda``), ops ``torch.ops.torchsoftdtw_refcu.forward/backward``:
  the GPU implementation the tests compare against on the same device.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (CPU baseline / reference arm) use it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle_softdtw.so")
REF_SO = os.path.join(HERE, "_ref", "libsoftdtw_ref_cpu.so")
REF_CUDA_SO = os.path.join(HERE, "_ref", "libsoftdtw_ref_cuda.so")

_lib = None
_ref_loaded = False
_ref_cuda_loaded = False

_i64 = ctypes.c_int64
_p = ctypes.c_void_p


def build() -> None:
    """Compile the C restatement (and the reference, when its sources are mounted)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if os.path.isdir("/root/reference/src"):
        subprocess.run(["make", "-s", "-C", HERE, "ref", "ref-cuda"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.oracle_in_band.restype = ctypes.c_int
        L.oracle_in_band.argtypes = [_i64, _i64, _i64, _i64, _i64]
        L.oracle_count_cells.restype = _i64
        L.oracle_count_cells.argtypes = [_p, _p, _i64, _i64]
        for suf in ("f32", "f64"):
            f = getattr(L, f"oracle_forward_{suf}")
            f.restype = None
            f.argtypes = [_p, _i64, _i64, _i64, _p, _p, ctypes.c_double, _i64, _p, _p, ctypes.c_int]
            g = getattr(L, f"oracle_backward_{suf}")
            g.restype = None
            g.argtypes = [_p, _p, _i64, _i64, _i64, _p, _p, ctypes.c_double, _i64, _p, ctypes.c_int]
        _lib = L
    return _lib


def default_threads() -> int:
    return max(1, os.cpu_count() or 1)


def _suffix(dtype) -> str:
    if dtype == np.float32:
        return "f32"
    if dtype == np.float64:
        return "f64"
    raise TypeError(f"oracle supports float32/float64, got {dtype}")


def _lengths(lx, B, default):
    if lx is None:
        return np.full((B,), default, dtype=np.int64)
    return np.ascontiguousarray(np.asarray(lx, dtype=np.int64))


def in_band(i: int, j: int, nx: int, ny: int, bandwidth: int) -> bool:
    return bool(lib().oracle_in_band(i, j, nx, ny, bandwidth))


def count_cells(lx, ly, bandwidth: int) -> int:
    lx = np.ascontiguousarray(np.asarray(lx, dtype=np.int64))
    ly = np.ascontiguousarray(np.asarray(ly, dtype=np.int64))
    return int(lib().oracle_count_cells(lx.ctypes.data, ly.ctypes.data, lx.shape[0], bandwidth))


def forward(D: np.ndarray, lx=None, ly=None, gamma: float = 1.0, bandwidth: int = -1, nthreads: int | None = None):
    """Reference forward: returns (costs (B,), R (B,N+2,M+2)) in D's dtype (float32/float64)."""
    D = np.ascontiguousarray(D)
    B, N, M = D.shape
    lx, ly = _lengths(lx, B, N), _lengths(ly, B, M)
    R = np.empty((B, N + 2, M + 2), dtype=D.dtype)
    costs = np.empty((B,), dtype=D.dtype)
    fn = getattr(lib(), f"oracle_forward_{_suffix(D.dtype)}")
    fn(D.ctypes.data, B, N, M, lx.ctypes.data, ly.ctypes.data, float(gamma), int(bandwidth),
       R.ctypes.data, costs.ctypes.data, int(nthreads or default_threads()))
    return costs, R


def backward(D: np.ndarray, R: np.ndarray, lx=None, ly=None, gamma: float = 1.0, bandwidth: int = -1,
             nthreads: int | None = None) -> np.ndarray:
    """Reference backward: returns E = d(costs)/dD (B,N,M) in D's dtype."""
    D = np.ascontiguousarray(D)
    R = np.ascontiguousarray(R, dtype=D.dtype)
    B, N, M = D.shape
    lx, ly = _lengths(lx, B, N), _lengths(ly, B, M)
    E = np.empty((B, N, M), dtype=D.dtype)
    fn = getattr(lib(), f"oracle_backward_{_suffix(D.dtype)}")
    fn(D.ctypes.data, R.ctypes.data, B, N, M, lx.ctypes.data, ly.ctypes.data, float(gamma), int(bandwidth),
       E.ctypes.data, int(nthreads or default_threads()))
    return E


def pairwise_l2_squared(X: np.ndarray, Y: np.ndarray) -> np.ndarray:
    """Restatement of the reference's distance (``src/torchsoftdtw/distances.py:4-18``) in numpy:
    |x|^2 + |y|^2 - 2 x.y, clamped at 0. Returns (D, mask) where mask = (unclamped D >= 0), the set of
    cells through which the clamp passes gradient."""
    x2 = (X * X).sum(-1)
    y2 = (Y * Y).sum(-1)
    xy = np.matmul(X, np.swapaxes(Y, 1, 2))
    Draw = x2[:, :, None] + y2[:, None, :] - 2 * xy
    return np.maximum(Draw, 0), Draw >= 0


def module_forward_backward(X, Y, lx=None, ly=None, gamma=1.0, bandwidth=-1, normalize=False, grad_out=None,
                            nthreads=None):
    """Restatement of the reference module path (``softdtw.py:106-142`` + autograd of ``distances.py:14-18``):
    returns (costs, grad_X, grad_Y) for loss = sum(grad_out * costs), computed in X's dtype."""
    B, N, _ = X.shape
    M = Y.shape[1]
    D, mask = pairwise_l2_squared(X, Y)
    D = D.astype(X.dtype)
    lx_, ly_ = _lengths(lx, B, N), _lengths(ly, B, M)
    costs, R = forward(D, lx_, ly_, gamma, bandwidth, nthreads)
    E = backward(D, R, lx_, ly_, gamma, bandwidth, nthreads)
    g = np.ones((B,), dtype=X.dtype) if grad_out is None else np.asarray(grad_out, dtype=X.dtype)
    if normalize:
        div = (lx_ + ly_ - 1).astype(X.dtype)
        costs = costs / div
        g = g / div
    G = g[:, None, None] * E * mask
    rs = G.sum(2)
    cs = G.sum(1)
    grad_X = 2 * (rs[:, :, None] * X - np.matmul(G, Y))
    grad_Y = 2 * (cs[:, :, None] * Y - np.matmul(np.swapaxes(G, 1, 2), X))
    return costs, grad_X.astype(X.dtype), grad_Y.astype(X.dtype)


# ----------------------------------------------------------------------------------------------------
# The compiled reference (torch ops in the `torchsoftdtw_ref` namespace)
# ----------------------------------------------------------------------------------------------------

def ref_available() -> bool:
    return os.path.exists(REF_SO)


def load_ref():
    """Load the compiled reference CPU operator; returns torch.ops.torchsoftdtw_ref."""
    global _ref_loaded
    import torch

    if not _ref_loaded:
        torch.ops.load_library(REF_SO)
        _ref_loaded = True
    return torch.ops.torchsoftdtw_ref


def load_ref_cuda():
    """Load the compiled reference CUDA operator; returns torch.ops.torchsoftdtw_refcu (its CPU kernels
    are registered too)."""
    global _ref_cuda_loaded
    import torch

    if not _ref_cuda_loaded:
        if not os.path.exists(REF_CUDA_SO):
            raise FileNotFoundError(f"{REF_CUDA_SO} is missing: build it with `make -C oracle ref-cuda`")
        torch.ops.load_library(REF_CUDA_SO)
        _ref_cuda_loaded = True
    return torch.ops.torchsoftdtw_refcu


# ----------------------------------------------------------------------------------------------------
# The reference's module path on its compiled CPU operator (bench.py's CPU baseline and reference arm).
# Nothing here imports torchsoftdtw_b200, so a process that runs only this path maps no library of the
# product.
# ----------------------------------------------------------------------------------------------------

def ref_pairwise_l2_squared_torch(X, Y):
    """Torch restatement of the reference's ``pairwise_l2_squared`` (``src/torchsoftdtw/distances.py:4-18``):
    |x|^2 + |y|^2 - 2 x.y through ``bmm``, clamped at 0; differentiable by torch autograd as in the
    reference's module."""
    import torch

    x2 = (X * X).sum(dim=-1)
    y2 = (Y * Y).sum(dim=-1)
    xy = torch.bmm(X, Y.transpose(1, 2))
    return (x2.unsqueeze(2) + y2.unsqueeze(1) - 2 * xy).clamp_min(0.0)


def _ref_autograd_class():
    import torch

    class RefSoftDTWAutograd(torch.autograd.Function):
        """The reference's ``SoftDTWAutograd`` glue (``softdtw.py:33-48``) over its compiled CPU operator."""

        @staticmethod
        def forward(ctx, D, lx, ly, gamma, bw):
            costs, R = load_ref().forward(D, lx, ly, gamma, bw)
            ctx.save_for_backward(D, R, lx, ly)
            ctx.gamma, ctx.bw = gamma, bw
            return costs

        @staticmethod
        def backward(ctx, g):
            D, R, lx, ly = ctx.saved_tensors
            E = load_ref().backward(D, R, lx, ly, ctx.gamma, ctx.bw)
            return g.unsqueeze(-1).unsqueeze(-1) * E, None, None, None, None

    return RefSoftDTWAutograd


_REF_AUTOGRAD = None


def reference_module_step(X, Y, lx, ly, gamma: float, bandwidth: int, normalize: bool, backward: bool = True):
    """One step of the reference module (``SoftDTW.forward``, ``softdtw.py:106-142``) on CPU tensors:
    the distance, the compiled reference operator under torch autograd, the optional normalisation,
    and (``backward``) grad_X of ``costs.sum()``. Returns (costs, grad_X or None)."""
    global _REF_AUTOGRAD
    if _REF_AUTOGRAD is None:
        _REF_AUTOGRAD = _ref_autograd_class()
    Xr = X.detach().requires_grad_(backward)
    D = ref_pairwise_l2_squared_torch(Xr, Y)
    costs = _REF_AUTOGRAD.apply(D, lx, ly, float(gamma), int(bandwidth))
    if normalize:
        costs = costs / (lx + ly - 1).to(costs.dtype)
    if backward:
        costs.sum().backward()
        return costs.detach(), Xr.grad
    return costs.detach(), None
