"""GPU: the runtime properties of the ops — torch.compile, CUDA-graph capture/replay, determinism,
concurrent streams, the C ABI called directly, and failure detection without a GPU fault:

* a wait that runs out (both kernel families, forward and backward): the failure-path hook makes one
  strip finish without publishing its progress; the next strip's bounded wait expires, the launch
  aborts, the host reads SDTW_ERR_TIMEOUT, and the context stays usable (a normal launch right after
  is correct);
* the strip-ticket and pair-resident kernels agree bit for bit; the pair-resident kernels are correct
  for any number of warps per CTA;
* lengths outside [0, N]: NaN cost and SDTW_ERR_BAD_LENGTH, no out-of-range access.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
import torchsoftdtw_b200 as T
from torchsoftdtw_b200 import _ext

pytestmark = pytest.mark.gpu


def test_torch_compile_matches_eager(cuda):
    torch.manual_seed(0)
    X = torch.randn(4, 30, 8, device=cuda)
    Y = torch.randn(4, 25, 8, device=cuda)
    D = torch.rand(4, 30, 25, device=cuda)
    m = T.SoftDTW(gamma=0.5, bandwidth=4, normalize=True)

    def f(x, y, d):
        return m(x, y).sum() + T.soft_dtw(d, gamma=0.3).sum()

    eager = f(X, Y, D)
    compiled = torch.compile(f)(X, Y, D)
    torch.testing.assert_close(compiled, eager, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("distance", ["l2_squared", "l1", "cosine"])
def test_torch_compile_module_fwd_bwd_matches_eager(cuda, distance):
    """Every module path (fused squared L2, L1, cosine) traces under torch.compile through the FakeTensor
    kernels, forward and backward, and matches eager."""
    torch.manual_seed(5)
    X = torch.randn(3, 20, 8, device=cuda)
    Y = torch.randn(3, 16, 8, device=cuda)
    m = T.SoftDTW(gamma=0.4, distance=distance)

    def f(x, y):
        return m(x, y).sum()

    Xe = X.clone().requires_grad_(True)
    Xc = X.clone().requires_grad_(True)
    eager = f(Xe, Y)
    eager.backward()
    compiled = torch.compile(f)(Xc, Y)
    compiled.backward()
    torch.testing.assert_close(compiled, eager, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(Xc.grad, Xe.grad, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("path", [0, 3])
def test_cuda_graph_module_step_replay(cuda, path):
    """A whole module step (cost matrix, forward, backward, gradient) captured in a CUDA graph and replayed on
    new inputs equals the eager step; path 3 forces the warp-per-pair wavefront kernels, and the fp64 d = 4
    inputs take the narrow cost and gradient kernels."""
    lib = _ext.capi()
    lib.sdtw_debug_force_path(path)
    try:
        torch.manual_seed(6)
        X = torch.randn(64, 40, 4, device=cuda, dtype=torch.float64, requires_grad=True)
        Y = torch.randn(64, 36, 4, device=cuda, dtype=torch.float64)
        m = T.SoftDTW(gamma=0.7)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up outside capture
                X.grad = None
                m(X, Y).sum().backward()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        X.grad = None
        with torch.cuda.graph(g):
            loss = m(X, Y).sum()
            loss.backward()
        for _ in range(2):
            with torch.no_grad():
                X.copy_(torch.randn_like(X))
                Y.copy_(torch.randn_like(Y))
            g.replay()
            torch.cuda.synchronize()
            Xr = X.detach().clone().requires_grad_(True)
            ref = m(Xr, Y).sum()
            ref.backward()
            torch.testing.assert_close(loss, ref, rtol=1e-12, atol=1e-12)
            torch.testing.assert_close(X.grad, Xr.grad, rtol=1e-12, atol=1e-12)
        del g
    finally:
        lib.sdtw_debug_force_path(0)


def test_cuda_graph_capture_and_replay(cuda):
    torch.manual_seed(1)
    D = torch.rand(8, 100, 90, device=cuda)
    lx = torch.full((8,), 100, device=cuda, dtype=torch.long)
    ly = torch.full((8,), 90, device=cuda, dtype=torch.long)
    costs, R = torch.ops.torchsoftdtw.forward(D, lx, ly, 0.5, 7)  # warm-up outside capture
    E = torch.ops.torchsoftdtw.backward(D, R, lx, ly, 0.5, 7)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            gc, gR = torch.ops.torchsoftdtw.forward(D, lx, ly, 0.5, 7)
            gE = torch.ops.torchsoftdtw.backward(D, gR, lx, ly, 0.5, 7)
    torch.cuda.current_stream().wait_stream(s)
    for trial in range(3):
        D.copy_(torch.rand(8, 100, 90, device=cuda))
        g.replay()
        torch.cuda.synchronize()
        c_ref, R_ref = torch.ops.torchsoftdtw.forward(D, lx, ly, 0.5, 7)
        E_ref = torch.ops.torchsoftdtw.backward(D, R_ref, lx, ly, 0.5, 7)
        assert torch.equal(gc, c_ref) and torch.equal(gE, E_ref)
    del g


def test_deterministic(cuda):
    torch.manual_seed(2)
    X = torch.randn(16, 200, 16, device=cuda, requires_grad=True)
    Y = torch.randn(16, 180, 16, device=cuda)
    outs = []
    for _ in range(2):
        X.grad = None
        c = T.SoftDTW(gamma=0.1)(X, Y)
        c.sum().backward()
        outs.append((c.detach().clone(), X.grad.clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_concurrent_streams(cuda):
    torch.manual_seed(3)
    Ds = [torch.rand(4, 70 + 10 * k, 64, device=cuda, dtype=torch.float64) for k in range(4)]
    streams = [torch.cuda.Stream() for _ in Ds]
    outs = [None] * len(Ds)
    torch.cuda.synchronize()
    for k, (D, s) in enumerate(zip(Ds, streams)):
        with torch.cuda.stream(s):
            outs[k] = T.soft_dtw(D, gamma=0.2)
    torch.cuda.synchronize()
    for D, c in zip(Ds, outs):
        ref, _ = O.forward(D.cpu().numpy(), None, None, 0.2, -1)
        np.testing.assert_allclose(c.cpu().numpy(), ref, rtol=1e-10, atol=1e-12)


def test_c_abi_direct_call(cuda):
    """The C ABI used without torch's op layer: plain device pointers, a caller-owned workspace."""
    lib = _ext.capi()
    torch.manual_seed(4)
    B, N, M = 3, 50, 41
    D = torch.rand(B, N, M, device=cuda, dtype=torch.float64)
    lx = torch.tensor([50, 44, 3], device=cuda, dtype=torch.int32)
    ly = torch.tensor([41, 41, 40], device=cuda, dtype=torch.int32)
    R = torch.empty(B, N + 2, M + 2, device=cuda, dtype=torch.float64)
    costs = torch.empty(B, device=cuda, dtype=torch.float64)
    E = torch.empty(B, N, M, device=cuda, dtype=torch.float64)
    err = torch.zeros(1, device=cuda, dtype=torch.int32)
    wsf = lib.sdtw_forward_workspace_bytes(B, N, M, 1)
    wsb = lib.sdtw_backward_workspace_bytes(B, N, M, 1)
    ws = torch.empty(max(wsf, wsb), device=cuda, dtype=torch.uint8)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    st = lib.sdtw_forward(1, p(D), B, N, M, p(lx), p(ly), 1, 0.4, 3, p(R), p(costs), p(ws), wsf, p(err), stream)
    assert st == 0, lib.sdtw_status_string(st)
    st = lib.sdtw_backward(1, p(D), p(R), B, N, M, p(lx), p(ly), 1, 0.4, 3, p(E), p(ws), wsb, p(err), stream)
    assert st == 0, lib.sdtw_status_string(st)
    assert lib.sdtw_read_error_word(p(err), stream) == 0
    cr, Rr = O.forward(D.cpu().numpy(), [50, 44, 3], [41, 41, 40], 0.4, 3)
    Er = O.backward(D.cpu().numpy(), Rr, [50, 44, 3], [41, 41, 40], 0.4, 3)
    np.testing.assert_allclose(costs.cpu().numpy(), cr, rtol=1e-10)
    np.testing.assert_allclose(E.cpu().numpy(), Er, rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("path,direction", [(1, "forward"), (2, "forward"), (2, "backward")])
def test_wait_timeout_is_reported_and_context_survives(cuda, path, direction):
    """Strip 0 of pair 0 never publishes its boundary row (strip-ticket kernels: ticket 0; pair-resident
    kernels: pair 0 * 4 strips + strip 0); the strip that depends on it runs into its bounded wait."""
    lib = _ext.capi()
    torch.manual_seed(5)
    D = torch.rand(2, 128, 64, device=cuda)  # 4 strips of 32 rows per pair
    lx = torch.full((2,), 128, device=cuda, dtype=torch.long)
    ly = torch.full((2,), 64, device=cuda, dtype=torch.long)
    T.check_errors(cuda)
    _, R = torch.ops.torchsoftdtw.forward(D, lx, ly, 1.0, -1)
    torch.cuda.synchronize()
    lib.sdtw_debug_force_path(path)
    lib.sdtw_set_wait_timeout(0.2)
    # backward: strip 0 is swept last and has no consumer; stall strip 3 (the first) instead
    lib.sdtw_debug_inject_stall(0 if direction == "forward" else 3)
    try:
        if direction == "forward":
            c, _ = torch.ops.torchsoftdtw.forward(D, lx, ly, 1.0, -1)
        else:
            torch.ops.torchsoftdtw.backward(D, R, lx, ly, 1.0, -1)
        torch.cuda.synchronize()
        if direction == "forward":
            # The aborted pair never reaches its terminal cell: its cost stays at the NaN it starts as, so
            # a caller that never reads the error word still cannot mistake it for a value.
            assert torch.isnan(c[0]).item()
        with pytest.raises(RuntimeError, match="timed out"):
            T.check_errors(cuda)
    finally:
        lib.sdtw_debug_inject_stall(-1)
        lib.sdtw_set_wait_timeout(2.0)
    try:
        costs = T.soft_dtw(D.double())
        ref, _ = O.forward(D.double().cpu().numpy(), None, None, 1.0, -1)
        np.testing.assert_allclose(costs.cpu().numpy(), ref, rtol=1e-10)
        T.check_errors(cuda)
    finally:
        lib.sdtw_debug_force_path(0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("B,N,M,bw,ragged", [(3, 100, 90, -1, False), (4, 257, 130, 20, True), (5, 64, 300, 3, True),
                                             (2, 31, 33, -1, True), (3, 450, 70, 0, False)])
def test_kernel_families_agree_bit_for_bit(cuda, dtype, B, N, M, bw, ragged):
    """The strip-ticket and pair-resident kernels evaluate every cell with the same expression in the
    same order, so costs, R and E agree exactly."""
    lib = _ext.capi()
    g = torch.Generator().manual_seed(N + M + B)
    D = (torch.rand(B, N, M, generator=g, dtype=torch.float64) * 2).to(dtype).to(cuda)
    if ragged:
        lx = torch.randint(max(1, N // 2), N + 1, (B,), generator=g)
        ly = torch.randint(max(1, M // 2), M + 1, (B,), generator=g)
    else:
        lx, ly = torch.full((B,), N), torch.full((B,), M)
    lx, ly = lx.to(cuda), ly.to(cuda)
    outs = []
    try:
        for path in (1, 2):
            lib.sdtw_debug_force_path(path)
            c, R = torch.ops.torchsoftdtw.forward(D, lx, ly, 0.3, bw)
            E = torch.ops.torchsoftdtw.backward(D, R, lx, ly, 0.3, bw)
            torch.cuda.synchronize()
            outs.append((c, R, E))
    finally:
        lib.sdtw_debug_force_path(0)
    T.check_errors(cuda)
    for x, y in zip(outs[0], outs[1]):
        assert torch.equal(x, y)


@pytest.mark.parametrize("warps", [1, 2, 3, 5, 16])
def test_pair_kernels_any_warp_count(cuda, warps):
    """The pair-resident kernels are correct for any number of warps per CTA (strips wrap around the
    warps several times when warps < strips)."""
    lib = _ext.capi()
    g = torch.Generator().manual_seed(warps)
    B, N, M = 3, 300, 120
    D = torch.rand(B, N, M, generator=g, dtype=torch.float64)
    lx = torch.tensor([300, 287, 150])
    ly = torch.tensor([120, 97, 120])
    try:
        lib.sdtw_debug_force_path(2)
        lib.sdtw_debug_set_pair_warps(warps)
        c, R = torch.ops.torchsoftdtw.forward(D.to(cuda), lx.to(cuda), ly.to(cuda), 0.7, 40)
        E = torch.ops.torchsoftdtw.backward(D.to(cuda), R, lx.to(cuda), ly.to(cuda), 0.7, 40)
        torch.cuda.synchronize()
    finally:
        lib.sdtw_debug_force_path(0)
        lib.sdtw_debug_set_pair_warps(16)
    T.check_errors(cuda)
    cr, Rr = O.forward(D.numpy(), lx.numpy(), ly.numpy(), 0.7, 40)
    Er = O.backward(D.numpy(), Rr, lx.numpy(), ly.numpy(), 0.7, 40)
    np.testing.assert_allclose(c.cpu().numpy(), cr, rtol=1e-10)
    np.testing.assert_allclose(R.cpu().numpy(), Rr, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(E.cpu().numpy(), Er, rtol=1e-10, atol=1e-12)


def test_bad_lengths_give_nan_and_error_bit(cuda):
    D = torch.rand(3, 10, 10, device=cuda, dtype=torch.float64)
    lx = torch.tensor([10, 11, 5], device=cuda)
    ly = torch.tensor([10, 10, -1], device=cuda)
    costs, R = torch.ops.torchsoftdtw.forward(D, lx, ly, 1.0, -1)
    c = costs.cpu().numpy()
    assert np.isfinite(c[0]) and np.isnan(c[1]) and np.isnan(c[2])
    with pytest.raises(RuntimeError, match="outside"):
        T.check_errors(cuda)
    T.check_errors(cuda)  # cleared


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("B,N,M,bw,ragged", [(3, 100, 90, -1, False), (4, 257, 130, 20, True), (5, 64, 300, 3, True),
                                             (2, 31, 33, -1, True), (3, 450, 70, 0, False), (2, 200, 512, -1, False)])
def test_r_tiles_match_padded_r(cuda, dtype, B, N, M, bw, ragged):
    """The module path's R tiles (sdtw_forward_tiles / sdtw_backward_tiles, pair-resident kernels) give the costs
    and E of the padded R, and every tile row holds the padded R's values in units of gamma ln 2 (the tiles
    path runs the dynamic program in those units, so the two agree to rounding: fp64 to 1e-10; fp32 costs to
    1e-5 relative, E to 2e-3 absolute, the size of one ulp of R ~ 1e2 divided by gamma = 0.3 and carried
    along a path)."""
    lib = _ext.capi()
    code = 1 if dtype == torch.float64 else 0
    g = torch.Generator().manual_seed(N * 3 + M + B)
    D = (torch.rand(B, N, M, generator=g, dtype=torch.float64) * 2).to(dtype).to(cuda)
    if ragged:
        lx = torch.randint(max(1, N // 2), N + 1, (B,), generator=g)
        ly = torch.randint(max(1, M // 2), M + 1, (B,), generator=g)
    else:
        lx, ly = torch.full((B,), N), torch.full((B,), M)
    lx, ly = lx.to(cuda), ly.to(cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    err = torch.zeros(1, device=cuda, dtype=torch.int32)
    ws = torch.empty(max(lib.sdtw_forward_workspace_bytes(B, N, M, code), lib.sdtw_backward_workspace_bytes(B, N, M, code)),
                     device=cuda, dtype=torch.uint8)
    try:
        lib.sdtw_debug_force_path(2)
        assert lib.sdtw_r_tiled(B, N, M, code) == 1
        S, NBt = (N + 31) // 32, (M + 31) // 32 + 1
        assert lib.sdtw_r_tiles_elems(B, N, M) == B * S * NBt * 1024
        Rt = torch.full((B, S, NBt, 32, 32), float("nan"), device=cuda, dtype=dtype)
        c1 = torch.empty(B, device=cuda, dtype=dtype)
        E1 = torch.empty(B, N, M, device=cuda, dtype=dtype)
        st = lib.sdtw_forward_tiles(code, p(D), B, N, M, p(lx), p(ly), 0, 0.3, bw, p(Rt), p(c1), p(ws), ws.numel(),
                                    p(err), stream)
        assert st == 0, lib.sdtw_status_string(st)
        st = lib.sdtw_backward_tiles(code, p(Rt), B, N, M, p(lx), p(ly), 0, 0.3, bw, p(E1), p(ws), ws.numel(), p(err),
                                     stream)
        assert st == 0, lib.sdtw_status_string(st)
        c2, R2 = torch.ops.torchsoftdtw.forward(D, lx, ly, 0.3, bw)
        E2 = torch.ops.torchsoftdtw.backward(D, R2, lx, ly, 0.3, bw)
        torch.cuda.synchronize()
    finally:
        lib.sdtw_debug_force_path(0)
    assert lib.sdtw_read_error_word(p(err), stream) == 0
    T.check_errors(cuda)
    if dtype == torch.float64:
        torch.testing.assert_close(c1, c2, rtol=1e-10, atol=1e-12)
        torch.testing.assert_close(E1, E2, rtol=1e-10, atol=1e-12)
    else:
        torch.testing.assert_close(c1, c2, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(E1, E2, rtol=0, atol=2e-3)
    # Tile rows against the padded R: tile (b, s, k)[l][x] = R[32 s + l][32 k + x - l - 1] log2(e) / gamma (padded
    # row +1, column +1) wherever the tile was written (NaN marks a tile the forward did not sweep).
    gl = 0.3 * math.log(2.0)
    rtol = 1e-10 if dtype == torch.float64 else 1e-5
    Rt_c, R2_c = Rt.cpu().double().numpy() * gl, R2.cpu().double().numpy()
    written = 0
    lgrid, xgrid = np.meshgrid(np.arange(32), np.arange(32), indexing="ij")
    for b in range(B):
        for s in range(S):
            rows = min(32, N - 32 * s)
            for k in range(NBt):
                tile = Rt_c[b, s, k]
                if np.isnan(tile).all():
                    continue
                written += 1
                c = 32 * k + xgrid - lgrid - 1
                sel = (lgrid < rows) & (c >= 0) & (c < M)
                want = R2_c[b, 32 * s + lgrid[sel] + 1, c[sel] + 1]
                got = tile[sel]
                assert np.array_equal(np.isinf(got), np.isinf(want)), (b, s, k)
                fin = np.isfinite(want)
                np.testing.assert_allclose(got[fin], want[fin], rtol=rtol, atol=1e-9)
    assert written > 0
