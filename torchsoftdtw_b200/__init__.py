"""torchsoftdtw_b200 — a B200-native (sm_100a) Soft-DTW operator with the API of angelo-ortiz/torchsoftdtw.

Public names match the reference's ``torchsoftdtw/__init__.py``; the ops are registered under the same
``torch.ops.torchsoftdtw`` namespace. All compute runs in this package's CUDA kernels (``lib/``).
"""

from . import _ext
from .distances import pairwise_cosine, pairwise_l1, pairwise_l2_squared
from .softdtw import SoftDTW, SoftDTWAutograd, soft_dtw

__all__ = [
    "SoftDTW",
    "SoftDTWAutograd",
    "check_errors",
    "pairwise_cosine",
    "pairwise_l1",
    "pairwise_l2_squared",
    "soft_dtw",
]


def check_errors(device=None) -> None:
    """Synchronise and raise RuntimeError if any kernel on ``device`` reported a device-side error
    since the last check (a strip wait that timed out, or a length outside [0, N] / [0, M]).
    Clears the error word."""
    import torch

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    bits = int(torch.ops.torchsoftdtw_b200.error_bits(torch.empty(0, device=dev)).item())
    if bits:
        what = []
        if bits & 1:
            what.append("a wait on a neighbouring strip timed out")
        if bits & 2:
            what.append("a length was outside [0, N] / [0, M]")
        raise RuntimeError(f"torchsoftdtw_b200 device error 0x{bits:x}: " + "; ".join(what))
