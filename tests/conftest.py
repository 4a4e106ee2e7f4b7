import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200); run with -m gpu")


def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def golden_names(prefix: str) -> list[str]:
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for GPU tests. A GPU test on a machine without CUDA fails (it is never skipped)."""
    import torch

    assert torch.cuda.is_available(), "GPU test selected (-m gpu) but no CUDA device is available"
    import torchsoftdtw_b200  # noqa: F401  (loads the native libraries)

    return torch.device("cuda", 0)


KERNEL_PATHS = {"auto": 0, "ticket": 1, "pair": 2, "warp": 3}


@pytest.fixture(params=list(KERNEL_PATHS))
def kernel_path(request):
    """Runs a GPU test once per wavefront kernel family: chosen by shape ("auto"), the strip-ticket
    kernels (strips claimed from a global counter, boundaries in global memory), the pair-resident
    kernels (one CTA per pair, boundaries in shared memory) and the warp-per-pair kernels (one warp per
    pair, strips in sequence, operands in global memory)."""
    from torchsoftdtw_b200 import _ext

    lib = _ext.capi()
    lib.sdtw_debug_force_path(KERNEL_PATHS[request.param])
    yield request.param
    lib.sdtw_debug_force_path(0)
