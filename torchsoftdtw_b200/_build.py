"""In-tree build of the native parts of torchsoftdtw_b200.

* ``lib/libsdtw_b200.so`` — the CUDA kernel library with the C ABI of ``include/sdtw_b200.h``,
  compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``), CUDA runtime linked
  statically so the library carries the runtime its kernels were built with.
* ``lib/libsdtw_b200_debug.so`` — the same library built with ``-DSDTW_DEBUG_BOUNDS``: the pair-resident
  wavefront kernels check every global access against its buffer and report one outside as the error bit 4
  (``SDTW_ERR_BOUNDS``) instead of performing it. A test build, loaded only through ctypes by the tests.
* ``_C<ext>.so`` — the PyTorch operator layer (``csrc/torch_ops.cpp``), compiled by the host C++
  compiler against libtorch and linked to ``lib/libsdtw_b200.so`` through ``$ORIGIN/lib``.

Both are rebuilt only when a source is newer than the output. Run ``python torchsoftdtw_b200/_build.py`` (as a
file: importing the package would load the libraries it builds).
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(PKG, "lib")
KERNEL_LIB = os.path.join(LIBDIR, "libsdtw_b200.so")
DEBUG_KERNEL_LIB = os.path.join(LIBDIR, "libsdtw_b200_debug.so")
OBJDIR = os.path.join(PKG, "_build")
DEBUG_OBJDIR = os.path.join(PKG, "_build", "debug_bounds")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> str:
    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if home and os.path.isdir(home):
        return home
    nvcc = shutil.which("nvcc")
    if nvcc:
        return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))
    return "/usr/local/cuda"


def ops_lib_path() -> str:
    return os.path.join(PKG, "_C" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print("[torchsoftdtw_b200 build]", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _extra_flags(src: str) -> list[str]:
    # The wavefront kernels spell out every fused multiply-add they use (fma()); no other product is
    # contracted, so the two kernel families (and both directions) round every cell identically.
    if os.path.basename(src) in ("sdtw_wavefront.cu", "sdtw_pairwave.cu", "sdtw_compensated.cu"):
        return ["--fmad=false"]
    return []


def build_kernels(force: bool = False, debug_bounds: bool = False) -> str:
    """nvcc: csrc/*.cu -> lib/libsdtw_b200.so (sm_100a); with debug_bounds, lib/libsdtw_b200_debug.so."""
    out = DEBUG_KERNEL_LIB if debug_bounds else KERNEL_LIB
    objdir = DEBUG_OBJDIR if debug_bounds else OBJDIR
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(objdir, exist_ok=True)
    nvcc = os.path.join(_cuda_home(), "bin", "nvcc")
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))) + [os.path.join(INCLUDE, "sdtw_b200.h")]
    defs = ["-DSDTW_DEBUG_BOUNDS"] if debug_bounds else []
    objs = []
    jobs = []
    for src in sources:
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers + [__file__]):
            jobs.append([nvcc, *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", *defs, *_extra_flags(src), "-Xcompiler",
                         "-fPIC", "-I" + INCLUDE, "-I" + CSRC, "-c", src, "-o", obj])
    if jobs:
        with ThreadPoolExecutor(max_workers=len(jobs)) as ex:
            list(ex.map(_run, jobs))
    if force or _stale(out, objs):
        _run([nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", out, *objs])
    return out


def build_ops(force: bool = False) -> str:
    """g++: csrc/torch_ops.cpp -> _C.so, linked to lib/libsdtw_b200.so."""
    import torch
    from torch.utils import cpp_extension

    out = ops_lib_path()
    src = os.path.join(CSRC, "torch_ops.cpp")
    deps = [src, os.path.join(INCLUDE, "sdtw_b200.h"), KERNEL_LIB]
    if not (force or _stale(out, deps)):
        return out
    torch_dir = os.path.dirname(torch.__file__)
    cuda_inc = os.path.join(_cuda_home(), "include")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cxx = os.environ.get("CXX", "g++")
    cmd = [cxx, "-O2", "-fPIC", "-shared", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-I" + INCLUDE, "-I" + cuda_inc]
    for inc in cpp_extension.include_paths():
        cmd.append("-I" + inc)
    cmd += [src, "-o", out, "-L" + LIBDIR, "-lsdtw_b200", "-Wl,-rpath,$ORIGIN/lib",
            "-L" + os.path.join(torch_dir, "lib"), "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-Wl,-rpath," + os.path.join(torch_dir, "lib")]
    _run(cmd)
    return out


def build(force: bool = False) -> None:
    build_kernels(force)
    build_ops(force)
    build_kernels(force, debug_bounds=True)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
