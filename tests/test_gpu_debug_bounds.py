"""GPU: the debug-bounds build (lib/libsdtw_b200_debug.so, compiled with SDTW_DEBUG_BOUNDS), in which the
pair-resident wavefront kernels check every global access against its buffer and report one outside as
SDTW_ERR_BOUNDS instead of performing it (a memory checker that cannot trap the GPU). Shapes chosen for the
edges of the kernels' index arithmetic (rows and columns not multiples of 32, one-row and one-column pairs,
ragged lengths, tight and wide bands, fp32 and fp64, padded R and R tiles): no access may fall outside, and
the results must equal the release library's bit for bit.
"""

import ctypes

import pytest
import torch

from torchsoftdtw_b200 import _ext

pytestmark = pytest.mark.gpu

SDTW_ERR_BOUNDS = 4

CASES = [(3, 100, 90, -1, True), (4, 257, 130, 20, True), (5, 64, 300, 3, True), (2, 31, 33, -1, True),
         (3, 450, 70, 0, False), (2, 200, 512, -1, False), (4, 1, 40, -1, True), (4, 40, 1, -1, True),
         (3, 193, 161, 7, True)]


def p(t):
    return ctypes.c_void_p(t.data_ptr())


def run(lib, D, lx, ly, bw, tiles, code):
    B, N, M = D.shape
    dev = D.device
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    err = torch.zeros(1, device=dev, dtype=torch.int32)
    ws = torch.empty(max(lib.sdtw_forward_workspace_bytes(B, N, M, code),
                         lib.sdtw_backward_workspace_bytes(B, N, M, code)), device=dev, dtype=torch.uint8)
    c = torch.empty(B, device=dev, dtype=D.dtype)
    E = torch.empty(B, N, M, device=dev, dtype=D.dtype)
    lib.sdtw_debug_force_path(2)
    try:
        if tiles:
            assert lib.sdtw_r_tiled(B, N, M, code) == 1
            R = torch.empty(lib.sdtw_r_tiles_elems(B, N, M), device=dev, dtype=D.dtype)
            st = lib.sdtw_forward_tiles(code, p(D), B, N, M, p(lx), p(ly), 0, 0.4, bw, p(R), p(c), p(ws), ws.numel(),
                                        p(err), stream)
            assert st == 0, lib.sdtw_status_string(st)
            st = lib.sdtw_backward_tiles(code, p(R), B, N, M, p(lx), p(ly), 0, 0.4, bw, p(E), p(ws), ws.numel(),
                                         p(err), stream)
        else:
            R = torch.empty(B, N + 2, M + 2, device=dev, dtype=D.dtype)
            st = lib.sdtw_forward(code, p(D), B, N, M, p(lx), p(ly), 0, 0.4, bw, p(R), p(c), p(ws), ws.numel(), p(err),
                                  stream)
            assert st == 0, lib.sdtw_status_string(st)
            st = lib.sdtw_backward(code, p(D), p(R), B, N, M, p(lx), p(ly), 0, 0.4, bw, p(E), p(ws), ws.numel(), p(err),
                                   stream)
        assert st == 0, lib.sdtw_status_string(st)
        torch.cuda.synchronize()
    finally:
        lib.sdtw_debug_force_path(0)
    bits = lib.sdtw_read_error_word(p(err), stream)
    return c, E, bits


@pytest.mark.parametrize("tiles", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("B,N,M,bw,ragged", CASES)
def test_no_access_outside_buffers(cuda, B, N, M, bw, ragged, dtype, tiles):
    code = 1 if dtype == torch.float64 else 0
    g = torch.Generator().manual_seed(B * 1000 + N + M)
    # D sits in the middle of a larger allocation, so that the bounds checks (not the allocator's padding)
    # decide what an access outside D would read.
    store = (torch.rand(3 * B * N * M + 64, generator=g, dtype=torch.float64) * 2).to(dtype).to(cuda)
    D = store[B * N * M + 7: 2 * B * N * M + 7].view(B, N, M)
    if ragged:
        lx = torch.randint(max(1, N // 2), N + 1, (B,), generator=g)
        ly = torch.randint(max(1, M // 2), M + 1, (B,), generator=g)
    else:
        lx, ly = torch.full((B,), N), torch.full((B,), M)
    lx, ly = lx.to(cuda), ly.to(cuda)
    c_dbg, E_dbg, bits = run(_ext.debug_capi(), D, lx, ly, bw, tiles, code)
    assert bits & SDTW_ERR_BOUNDS == 0, "a kernel access fell outside its buffer"
    assert bits == 0
    c_rel, E_rel, bits_rel = run(_ext.capi(), D, lx, ly, bw, tiles, code)
    assert bits_rel == 0
    assert torch.equal(c_dbg, c_rel)
    assert torch.equal(E_dbg, E_rel)


FUSED_CASES = [(148, 192, 200, 16, -1, False), (40, 256, 384, 48, 40, True), (20, 500, 130, 128, -1, True),
               (150, 193, 161, 32, 7, True)]


def run_fused(lib, X, Y, lx, ly, bw):
    B, N, d = X.shape
    M = Y.shape[1]
    dev = X.device
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    err = torch.zeros(1, device=dev, dtype=torch.int32)
    ws = torch.empty(lib.sdtw_forward_workspace_bytes(B, N, M, 0), device=dev, dtype=torch.uint8)
    c = torch.empty(B, device=dev)
    R = torch.full((lib.sdtw_r_tiles_elems(B, N, M),), float("nan"), device=dev)
    mask = torch.empty(lib.sdtw_clamp_mask_words(B, N, M), device=dev, dtype=torch.int32)
    flags = torch.empty(B, device=dev, dtype=torch.int32)
    assert lib.sdtw_forward_l2_fused_ok(B, N, M, d) == 1
    st = lib.sdtw_forward_l2_tiles(p(X), p(Y), B, N, M, d, p(lx), p(ly), 0, 0.4, bw, p(R), p(c), p(mask), p(flags),
                                   p(ws), ws.numel(), p(err), stream)
    assert st == 0, lib.sdtw_status_string(st)
    torch.cuda.synchronize()
    return c, R, mask, lib.sdtw_read_error_word(p(err), stream)


@pytest.mark.parametrize("B,N,M,d,bw,ragged", FUSED_CASES)
def test_fused_cost_forward_no_access_outside_buffers(cuda, B, N, M, d, bw, ragged):
    """The fused cost forward (cost tiles from X and Y inside the wavefront) under the same checks: X and Y sit
    inside larger allocations, rows past N and columns past M are read as clamped rows of the matrix."""
    g = torch.Generator().manual_seed(N * 7 + M + d)
    xs = torch.randn(3 * B * N * d + 64, generator=g).to(cuda)
    ys = torch.randn(3 * B * M * d + 64, generator=g).to(cuda)
    X = xs[B * N * d + 4: 2 * B * N * d + 4].view(B, N, d)  # 16-byte aligned: offsets are multiples of 4 floats
    Y = ys[B * M * d + 4: 2 * B * M * d + 4].view(B, M, d)
    if ragged:
        lx = torch.randint(max(1, N // 2), N + 1, (B,), generator=g)
        ly = torch.randint(max(1, M // 2), M + 1, (B,), generator=g)
    else:
        lx, ly = torch.full((B,), N), torch.full((B,), M)
    lx, ly = lx.to(cuda), ly.to(cuda)
    c_dbg, R_dbg, m_dbg, bits = run_fused(_ext.debug_capi(), X, Y, lx, ly, bw)
    assert bits & SDTW_ERR_BOUNDS == 0, "a kernel access fell outside its buffer"
    assert bits == 0
    c_rel, R_rel, m_rel, bits_rel = run_fused(_ext.capi(), X, Y, lx, ly, bw)
    assert bits_rel == 0
    assert torch.equal(c_dbg, c_rel)
    assert torch.equal(R_dbg.nan_to_num(7.0), R_rel.nan_to_num(7.0))
    assert torch.equal(m_dbg, m_rel)
