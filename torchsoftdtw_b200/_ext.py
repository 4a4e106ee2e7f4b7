"""Loader of the native libraries.

* ``_C`` (the PyTorch operator layer) is loaded with ``torch.ops.load_library``; it registers
  ``torch.ops.torchsoftdtw.forward/backward`` (the reference's schemas) and
  ``torch.ops.torchsoftdtw_b200.*`` (the fused squared-L2 module path).
* ``lib/libsdtw_b200.so`` (the CUDA kernels) is reachable directly through ctypes with :func:`capi`,
  which declares every entry point of ``include/sdtw_b200.h``.

There is no fallback: importing the package fails loudly when the libraries are not built.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _build

_loaded = False
_capi = None


def load() -> None:
    global _loaded
    if _loaded:
        return
    missing = [p for p in (_build.KERNEL_LIB, _build.ops_lib_path()) if not os.path.exists(p)]
    if missing:
        raise ImportError(
            "torchsoftdtw_b200: native libraries are not built (missing: "
            + ", ".join(missing)
            + "). Build them with `python torchsoftdtw_b200/_build.py` (needs nvcc for sm_100a)."
        )
    torch.ops.load_library(_build.ops_lib_path())
    _loaded = True


def library_paths() -> list[str]:
    """The native libraries this package loads (kernel library first)."""
    return [_build.KERNEL_LIB, _build.ops_lib_path()]


# Exported C-ABI symbols and their ctypes signatures (include/sdtw_b200.h).
_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_i = ctypes.c_int
_d = ctypes.c_double
_sz = ctypes.c_size_t
SIGNATURES: dict[str, tuple] = {
    "sdtw_status_string": (ctypes.c_char_p, [_i]),
    "sdtw_band_row_range": (None, [_i64, _i64, _i64, _i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "sdtw_pair_cells": (_i64, [_i64, _i64, _i64]),
    "sdtw_read_error_word": (ctypes.c_uint32, [_p, _p]),
    "sdtw_set_wait_timeout": (None, [_d]),
    "sdtw_forward_workspace_bytes": (_sz, [_i64, _i64, _i64, _i]),
    "sdtw_forward": (_i, [_i, _p, _i64, _i64, _i64, _p, _p, _i, _d, _i64, _p, _p, _p, _sz, _p, _p]),
    "sdtw_forward_band_r": (_i, [_i, _p, _i64, _i64, _i64, _p, _p, _i, _d, _i64, _p, _p, _p, _sz, _p, _p]),
    "sdtw_forward_noalloc": (_i, [_i, _p, _i64, _i64, _i64, _p, _p, _i, _d, _i64, _p, _p, _p, _p]),
    "sdtw_backward_workspace_bytes": (_sz, [_i64, _i64, _i64, _i]),
    "sdtw_backward": (_i, [_i, _p, _p, _i64, _i64, _i64, _p, _p, _i, _d, _i64, _p, _p, _sz, _p, _p]),
    "sdtw_r_tiled": (_i, [_i64, _i64, _i64, _i]),
    "sdtw_r_tiles_elems": (_i64, [_i64, _i64, _i64]),
    "sdtw_forward_tiles": (_i, [_i, _p, _i64, _i64, _i64, _p, _p, _i, _d, _i64, _p, _p, _p, _sz, _p, _p]),
    "sdtw_backward_tiles": (_i, [_i, _p, _i64, _i64, _i64, _p, _p, _i, _d, _i64, _p, _p, _sz, _p, _p]),
    "sdtw_forward_l2_fused_ok": (_i, [_i64, _i64, _i64, _i64]),
    "sdtw_clamp_mask_words": (_i64, [_i64, _i64, _i64]),
    "sdtw_forward_l2_tiles": (_i, [_p, _p, _i64, _i64, _i64, _i64, _p, _p, _i, _d, _i64, _p, _p, _p, _p, _p, _sz, _p,
                                   _p]),
    "sdtw_apply_clamp_mask": (_i, [_p, _p, _p, _i64, _i64, _i64, _p]),
    "sdtw_forward_x2": (_i, [_p, _i64, _i64, _i64, _p, _p, _i, _d, _i64, _p, _p, _p, _p, _p]),
    "sdtw_backward_x2": (_i, [_p, _p, _i64, _i64, _i64, _p, _p, _i, _d, _i64, _p, _p, _p]),
    "sdtw_pairwise_l2": (_i, [_i, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "sdtw_grad_l2": (_i, [_i, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "sdtw_pairwise_l2_band_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "sdtw_pairwise_l2_band": (_i, [_i, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _i, _i64, _p, _p, _p, _sz, _p]),
    "sdtw_grad_l2_band": (_i, [_i, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _i, _i64, _p, _p, _p]),
    "sdtw_pairwise_dist": (_i, [_i, _i, _p, _p, _i64, _i64, _i64, _i64, _d, _p, _p]),
    "sdtw_grad_dist_workspace_bytes": (_sz, [_i64, _i64, _i]),
    "sdtw_grad_dist": (_i, [_i, _i, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _d, _p, _p, _p, _p]),
}
# Test and tuning hooks (declared in the .cu, not part of the public header).
DEBUG_SIGNATURES: dict[str, tuple] = {
    "sdtw_debug_inject_stall": (None, [_i]),
    "sdtw_debug_force_path": (None, [_i]),
    "sdtw_debug_set_pair_warps": (None, [_i]),
    "sdtw_debug_kernel_launches": (ctypes.c_uint64, []),
    "sdtw_debug_force_distance_path": (None, [_i]),
}


def _declare(path: str) -> ctypes.CDLL:
    lib = ctypes.CDLL(path)
    for name, (res, args) in {**SIGNATURES, **DEBUG_SIGNATURES}.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def capi() -> ctypes.CDLL:
    """ctypes handle of lib/libsdtw_b200.so with every C-ABI signature declared."""
    global _capi
    if _capi is None:
        if not os.path.exists(_build.KERNEL_LIB):
            raise ImportError(f"torchsoftdtw_b200: {_build.KERNEL_LIB} is not built")
        _capi = _declare(_build.KERNEL_LIB)
    return _capi


_debug_capi = None


def debug_capi() -> ctypes.CDLL:
    """ctypes handle of lib/libsdtw_b200_debug.so, the build whose pair-resident kernels check every global
    access against its buffer (SDTW_ERR_BOUNDS instead of the access). For tests; nothing else loads it."""
    global _debug_capi
    if _debug_capi is None:
        if not os.path.exists(_build.DEBUG_KERNEL_LIB):
            raise ImportError(f"torchsoftdtw_b200: {_build.DEBUG_KERNEL_LIB} is not built")
        _debug_capi = _declare(_build.DEBUG_KERNEL_LIB)
    return _debug_capi


def r_tiled(B: int, N: int, M: int, dtype: torch.dtype, device) -> bool:
    """Whether the module path keeps R as the forward's strip tiles for this shape and dtype on ``device``
    (include/sdtw_b200.h, sdtw_r_tiled)."""
    if B <= 0 or N <= 0 or M <= 0 or dtype not in (torch.float32, torch.float64):
        return False
    dev = torch.device(device)
    if dev.type != "cuda":
        return False
    with torch.cuda.device(dev):
        return bool(capi().sdtw_r_tiled(B, N, M, 1 if dtype == torch.float64 else 0))


FUSED_COST_ENV = "TORCHSOFTDTW_B200_FUSED_COST"


def l2_fused(B: int, N: int, M: int, d: int, dtype: torch.dtype, device) -> bool:
    """Whether ``torchsoftdtw_b200::l2_forward`` computes the cost matrix inside the forward wavefront
    (sdtw_forward_l2_tiles) instead of storing it: only with ``TORCHSOFTDTW_B200_FUSED_COST=1`` in the
    environment, for fp32 shapes the library accepts (sdtw_forward_l2_fused_ok). The op's third output is
    then the clamp mask in place of D. The op layer reads the same variable on every call."""
    if os.environ.get(FUSED_COST_ENV, "0") in ("", "0") or dtype != torch.float32:
        return False
    if B <= 0 or N <= 0 or M <= 0 or d <= 0:
        return False
    dev = torch.device(device)
    if dev.type != "cuda":
        return False
    with torch.cuda.device(dev):
        return bool(capi().sdtw_forward_l2_fused_ok(B, N, M, d))
