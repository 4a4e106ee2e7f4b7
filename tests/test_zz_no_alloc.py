"""GPU: sdtw_forward_noalloc, the forward that uses the library's static device scratch instead of a
caller workspace, called through the C ABI and compared with sdtw_forward on the same inputs.

This file is collected last on purpose: the first sdtw_forward_noalloc call of a process looks its scratch
up, and the tests must pass both in a fresh process (this file alone) and after every other GPU test.
"""

import ctypes

import pytest
import torch

from torchsoftdtw_b200 import _ext

pytestmark = pytest.mark.gpu

SDTW_ETOOLARGE = -5


def p(t):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def inputs(B, N, M, dtype, ragged, dev, seed):
    g = torch.Generator().manual_seed(seed)
    D = (torch.rand(B, N, M, generator=g, dtype=torch.float64) * 3).to(dtype).to(dev)
    if ragged:
        lx = torch.randint(max(1, N // 2), N + 1, (B,), generator=g)
        ly = torch.randint(max(1, M // 2), M + 1, (B,), generator=g)
    else:
        lx, ly = torch.full((B,), N), torch.full((B,), M)
    return D, lx.to(dev), ly.to(dev)


def forward_workspace(lib, D, lx, ly, gamma, bw, code):
    B, N, M = D.shape
    R = torch.empty(B, N + 2, M + 2, device=D.device, dtype=D.dtype)
    c = torch.empty(B, device=D.device, dtype=D.dtype)
    err = torch.zeros(1, device=D.device, dtype=torch.int32)
    n = lib.sdtw_forward_workspace_bytes(B, N, M, code)
    ws = torch.empty(n, device=D.device, dtype=torch.uint8)
    st = lib.sdtw_forward(code, p(D), B, N, M, p(lx), p(ly), 0, gamma, bw, p(R), p(c), p(ws), n, p(err), stream())
    assert st == 0, lib.sdtw_status_string(st)
    torch.cuda.synchronize()
    assert lib.sdtw_read_error_word(p(err), stream()) == 0
    return c, R


def forward_noalloc(lib, D, lx, ly, gamma, bw, code):
    B, N, M = D.shape
    R = torch.empty(B, N + 2, M + 2, device=D.device, dtype=D.dtype)
    c = torch.empty(B, device=D.device, dtype=D.dtype)
    err = torch.zeros(1, device=D.device, dtype=torch.int32)
    st = lib.sdtw_forward_noalloc(code, p(D), B, N, M, p(lx), p(ly), 0, gamma, bw, p(R), p(c), p(err), stream())
    assert st == 0, lib.sdtw_status_string(st)
    torch.cuda.synchronize()
    assert lib.sdtw_read_error_word(p(err), stream()) == 0
    return c, R


# (B, N, M, bandwidth, dtype, ragged): the headline shape (one CTA per pair), a small banded ragged batch
# (strips claimed from the ticket counter, boundary rows in the scratch), fp64, and the fp64 headline
# shape, which runs on the pair-resident kernels and needs only the scratch's header.
CASES = [(256, 512, 512, -1, torch.float32, False), (6, 300, 200, 20, torch.float32, True),
         (4, 100, 90, -1, torch.float64, True), (256, 512, 512, -1, torch.float64, False)]


@pytest.mark.parametrize("B,N,M,bw,dtype,ragged", CASES)
def test_noalloc_forward_matches_workspace_forward_twice(cuda, B, N, M, bw, dtype, ragged):
    lib = _ext.capi()
    code = 1 if dtype == torch.float64 else 0
    tol = dict(rtol=1e-12, atol=1e-12) if dtype == torch.float64 else dict(rtol=1e-6, atol=1e-6)
    D, lx, ly = inputs(B, N, M, dtype, ragged, cuda, seed=B + N + M)
    c_ref, R_ref = forward_workspace(lib, D, lx, ly, 0.5, bw, code)
    for _ in range(2):  # two calls in a row reuse the same scratch
        c, R = forward_noalloc(lib, D, lx, ly, 0.5, bw, code)
        torch.testing.assert_close(c, c_ref, **tol)
        torch.testing.assert_close(R, R_ref, **tol)


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    lib = _ext.capi()
    # Few long pairs run on the strip-ticket kernels: 16 pairs * 128 strips * 4096 * 4 bytes of boundary
    # rows (32 MiB) > 16 MiB.
    B, N, M = 16, 4096, 4096
    assert lib.sdtw_forward_workspace_bytes(B, N, M, 0) > (16 << 20)
    dummy = torch.zeros(8, device=cuda)
    st = lib.sdtw_forward_noalloc(0, p(dummy), B, N, M, p(dummy), p(dummy), 0, 1.0, -1, p(dummy), p(dummy),
                                  p(dummy), stream())
    assert st == SDTW_ETOOLARGE
    assert b"static scratch" in lib.sdtw_status_string(st)
