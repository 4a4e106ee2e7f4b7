"""GPU: the band-restricted cost and gradient of the module path (sdtw_pairwise_l2_band, sdtw_grad_l2_band).

* sdtw_pairwise_l2_band writes, bit for bit, the same value as sdtw_pairwise_l2 into every cell of the region
  the dynamic program reads (rows below lengths_x, columns below lengths_y, inside the band), and leaves
  tiles that hold none of it unwritten;
* the forward and backward operators give bit-identical costs, R and E on either cost matrix;
* sdtw_grad_l2_band on the restricted cost matrix equals sdtw_grad_l2 on the full one (grad_X and grad_Y,
  with and without clamp flags);
* the SoftDTW module with a band is as accurate as the fp32 operator chain on the full cost matrix;
* lengths_x and lengths_y of different integer types are read as their values.
"""

import ctypes

import numpy as np
import pytest
import torch

import torchsoftdtw_b200 as T
from torchsoftdtw_b200 import _ext

pytestmark = pytest.mark.gpu

p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def region_mask(lx, ly, N, M, bw):
    lib = _ext.capi()
    mask = np.zeros((len(lx), N, M), dtype=bool)
    lo, hi = ctypes.c_int64(), ctypes.c_int64()
    for b, (nx, ny) in enumerate(zip(lx, ly)):
        for i in range(nx):
            lib.sdtw_band_row_range(i, nx, ny, bw, ctypes.byref(lo), ctypes.byref(hi))
            if lo.value <= hi.value:
                mask[b, i, lo.value:hi.value + 1] = True
    return torch.from_numpy(mask)


def pairwise_full(X, Y):
    lib = _ext.capi()
    B, N, d = X.shape
    M = Y.shape[1]
    D = torch.empty(B, N, M, device=X.device)
    fl = torch.empty(B, device=X.device, dtype=torch.int32)
    st = lib.sdtw_pairwise_l2(0, p(X), p(Y), B, N, M, d, p(D), p(fl), stream())
    assert st == 0, lib.sdtw_status_string(st)
    return D, fl


def pairwise_band(X, Y, lx, ly, bw):
    lib = _ext.capi()
    B, N, d = X.shape
    M = Y.shape[1]
    D = torch.full((B, N, M), float("nan"), device=X.device)
    fl = torch.empty(B, device=X.device, dtype=torch.int32)
    wsb = lib.sdtw_pairwise_l2_band_workspace_bytes(B, N, M)
    ws = torch.empty(wsb, device=X.device, dtype=torch.uint8)
    st = lib.sdtw_pairwise_l2_band(0, p(X), p(Y), B, N, M, d, p(lx), p(ly), int(lx.dtype == torch.int32), bw, p(D),
                                   p(fl), p(ws), wsb, stream())
    assert st == 0, lib.sdtw_status_string(st)
    return D, fl


def grad(X, Y, D, E, g, flags, band=None):
    lib = _ext.capi()
    B, N, d = X.shape
    M = Y.shape[1]
    gX, gY = torch.empty_like(X), torch.empty_like(Y)
    if band is None:
        st = lib.sdtw_grad_l2(0, p(X), p(Y), p(D), p(E), p(g), p(flags), B, N, M, d, p(gX), p(gY), stream())
    else:
        lx, ly, bw = band
        st = lib.sdtw_grad_l2_band(0, p(X), p(Y), p(D), p(E), p(g), p(flags), B, N, M, d, p(lx), p(ly),
                                   int(lx.dtype == torch.int32), bw, p(gX), p(gY), stream())
    assert st == 0, lib.sdtw_status_string(st)
    return gX, gY


# (B, N, M, d, bandwidth, lengths): lengths None = full; a list gives lengths_x and lengths_y per pair.
CASES = [
    (2, 1000, 1000, 32, 128, None),
    (3, 700, 520, 64, 40, ([700, 433, 90], [520, 517, 301])),
    (4, 300, 260, 16, 0, ([300, 0, 129, 7], [260, 260, 1, 9])),
    (2, 257, 384, 8, 5, ([257, 200], [384, 131])),
    (2, 640, 200, 64, 1000, ([640, 500], [200, 77])),
    (2, 150, 130, 12, 20, ([150, 149], [130, 66])),  # M % 4 != 0: the full cost matrix is computed
    (1, 4096, 4096, 16, 256, None),
]


@pytest.mark.parametrize("B,N,M,d,bw,lengths", CASES)
@pytest.mark.parametrize("ltype", [torch.int64, torch.int32])
def test_band_cost_and_gradient_match_the_full_ones(cuda, B, N, M, d, bw, lengths, ltype):
    g = torch.Generator().manual_seed(N * 7 + M + d + bw)
    X = torch.randn(B, N, d, generator=g).to(cuda)
    Y = torch.randn(B, M, d, generator=g).to(cuda)
    if lengths is None:
        lx_l, ly_l = [N] * B, [M] * B
    else:
        lx_l, ly_l = lengths
    lx = torch.tensor(lx_l, dtype=ltype, device=cuda)
    ly = torch.tensor(ly_l, dtype=ltype, device=cuda)
    Df, ff = pairwise_full(X, Y)
    Db, fb = pairwise_band(X, Y, lx, ly, bw)
    torch.cuda.synchronize()
    mask = region_mask(lx_l, ly_l, N, M, bw).to(cuda)
    assert torch.equal(Db[mask].view(torch.int32), Df[mask].view(torch.int32))
    # Flags: set for every pair with a clamped cell in the region, never for a pair without any.
    clamped = (Df.view(torch.int32) == -2147483648) & mask
    assert torch.all((fb != 0).int() >= clamped.flatten(1).any(1).int())
    assert torch.all((fb != 0).int() <= (ff != 0).int())
    if bw == 128 and N == 1000:
        assert torch.isnan(Db[:, :128, 896:]).all(), "tiles outside the band were written"

    gamma = 0.1
    cf, Rf = torch.ops.torchsoftdtw.forward(Df, lx, ly, gamma, bw)
    cb, Rb = torch.ops.torchsoftdtw.forward(Db, lx, ly, gamma, bw)
    assert torch.equal(cf, cb)
    assert torch.equal(Rf, Rb)
    E = torch.ops.torchsoftdtw.backward(Df, Rf, lx, ly, gamma, bw)
    Eb = torch.ops.torchsoftdtw.backward(Db, Rb, lx, ly, gamma, bw)
    assert torch.equal(E, Eb)
    assert torch.all(E[~mask] == 0)

    gc = torch.rand(B, generator=g).to(cuda) + 0.5
    for flags_f, flags_b in ((ff, fb), (None, None)):
        gXf, gYf = grad(X, Y, Df, E, gc, flags_f)
        gXb, gYb = grad(X, Y, Db, E, gc, flags_b, band=(lx, ly, bw))
        torch.cuda.synchronize()
        assert torch.isfinite(gXb).all() and torch.isfinite(gYb).all()
        assert torch.equal(gXf, gXb)
        assert torch.equal(gYf, gYb)


@pytest.mark.parametrize("bw", [16, 100])
def test_module_with_band_is_as_accurate_as_the_full_chain(cuda, bw):
    """The module (band-restricted cost and gradient) against the fp64 chain, within the error of the fp32
    operator chain on the full cost matrix (fp32 gradients are ill-conditioned at this scale of D; the bound
    is the unrestricted fp32 computation's own error, with a margin)."""
    B, N, M, d = 3, 600, 520, 64
    g = torch.Generator().manual_seed(bw)
    X = torch.randn(B, N, d, generator=g).to(cuda).requires_grad_(True)
    Y = torch.randn(B, M, d, generator=g).to(cuda).requires_grad_(True)
    lx = torch.tensor([600, 411, 23], device=cuda)
    ly = torch.tensor([520, 498, 30], device=cuda)
    loss = T.SoftDTW(gamma=0.5, bandwidth=bw)(X, Y, lengths_x=lx, lengths_y=ly)
    loss.sum().backward()
    # fp64 truth: the operators on the fp64 cost matrix, autograd through the cost.
    Xd, Yd = X.detach().double().requires_grad_(True), Y.detach().double().requires_grad_(True)
    D = ((Xd * Xd).sum(-1)[:, :, None] + (Yd * Yd).sum(-1)[:, None, :] - 2 * Xd @ Yd.transpose(1, 2)).clamp_min(0)
    c, R = torch.ops.torchsoftdtw.forward(D.detach(), lx, ly, 0.5, bw)
    E = torch.ops.torchsoftdtw.backward(D.detach(), R, lx, ly, 0.5, bw)
    (D * E).sum().backward()
    # The fp32 operator chain on the full cost matrix.
    Xf, Yf = X.detach(), Y.detach()
    Df, ff = pairwise_full(Xf, Yf)
    cf, Rf = torch.ops.torchsoftdtw.forward(Df, lx, ly, 0.5, bw)
    Ef = torch.ops.torchsoftdtw.backward(Df, Rf, lx, ly, 0.5, bw)
    gXf, gYf = grad(Xf, Yf, Df, Ef, torch.ones(B, device=cuda), ff)
    torch.cuda.synchronize()
    torch.testing.assert_close(loss.detach().double(), c, rtol=1e-5, atol=1e-3)
    for ours, chain, truth in ((X.grad, gXf, Xd.grad), (Y.grad, gYf, Yd.grad)):
        err = (ours.double() - truth).abs().max().item()
        err_chain = (chain.double() - truth).abs().max().item()
        assert err <= 2 * err_chain + 1e-5, (err, err_chain)


def test_mixed_length_dtypes_are_read_as_values(cuda):
    g = torch.Generator().manual_seed(3)
    D = torch.rand(3, 50, 40, generator=g).to(cuda)
    lx64 = torch.tensor([50, 31, 7], device=cuda)
    ly64 = torch.tensor([40, 12, 40], device=cuda)
    c0, R0 = torch.ops.torchsoftdtw.forward(D, lx64, ly64, 1.0, -1)
    c1, R1 = torch.ops.torchsoftdtw.forward(D, lx64.int(), ly64, 1.0, -1)
    c2, R2 = torch.ops.torchsoftdtw.forward(D, lx64, ly64.int(), 1.0, -1)
    assert torch.equal(c0, c1) and torch.equal(c0, c2)
    assert torch.equal(R0, R1) and torch.equal(R0, R2)
    E0 = torch.ops.torchsoftdtw.backward(D, R0, lx64, ly64, 1.0, -1)
    E1 = torch.ops.torchsoftdtw.backward(D, R0, lx64.int(), ly64, 1.0, -1)
    assert torch.equal(E0, E1)


def forward_c(D, lx, ly, gamma, bw, band_r):
    lib = _ext.capi()
    B, N, M = D.shape
    code = 1 if D.dtype == torch.float64 else 0
    R = torch.full((B, N + 2, M + 2), float("nan"), device=D.device, dtype=D.dtype)
    costs = torch.empty(B, device=D.device, dtype=D.dtype)
    wsb = max(lib.sdtw_forward_workspace_bytes(B, N, M, code), lib.sdtw_backward_workspace_bytes(B, N, M, code))
    ws = torch.empty(wsb, device=D.device, dtype=torch.uint8)
    err = torch.zeros(1, device=D.device, dtype=torch.int32)
    fn = lib.sdtw_forward_band_r if band_r else lib.sdtw_forward
    st = fn(code, p(D), B, N, M, p(lx), p(ly), int(lx.dtype == torch.int32), gamma, bw, p(R), p(costs), p(ws), wsb,
            p(err), stream())
    assert st == 0, lib.sdtw_status_string(st)
    E = torch.empty(B, N, M, device=D.device, dtype=D.dtype)
    st = lib.sdtw_backward(code, p(D), p(R), B, N, M, p(lx), p(ly), int(lx.dtype == torch.int32), gamma, bw, p(E),
                           p(ws), wsb, p(err), stream())
    assert st == 0, lib.sdtw_status_string(st)
    assert lib.sdtw_read_error_word(p(err), stream()) == 0
    return costs, R, E


# (B, N, M, bandwidth, lengths, dtype)
BAND_R_CASES = [
    (3, 300, 280, 20, ([300, 211, 64], [280, 280, 33]), torch.float32),
    (2, 1000, 900, -1, ([1000, 517], [900, 899]), torch.float32),
    (2, 130, 64, 0, ([130, 31], [64, 64]), torch.float64),
    (1, 2048, 2048, 128, None, torch.float32),
    (4, 97, 200, 7, ([97, 0, 96, 33], [200, 200, 1, 150]), torch.float64),
]


@pytest.mark.parametrize("B,N,M,bw,lengths,dtype", BAND_R_CASES)
def test_forward_band_r_feeds_the_backward_the_same_r(cuda, kernel_path, B, N, M, bw, lengths, dtype):
    """sdtw_forward_band_r leaves R unwritten outside what the backward reads: the costs and the backward's E
    equal sdtw_forward's, bit for bit, on every kernel family."""
    g = torch.Generator().manual_seed(N + M + B)
    D = (torch.rand(B, N, M, generator=g, dtype=torch.float64) * 2).to(dtype).to(cuda)
    lx_l, ly_l = lengths if lengths is not None else ([N] * B, [M] * B)
    lx = torch.tensor(lx_l, device=cuda)
    ly = torch.tensor(ly_l, device=cuda)
    c0, R0, E0 = forward_c(D, lx, ly, 0.3, bw, False)
    c1, R1, E1 = forward_c(D, lx, ly, 0.3, bw, True)
    torch.cuda.synchronize()
    assert torch.equal(c0.nan_to_num(), c1.nan_to_num())
    assert torch.equal(E0, E1)
    # In-band cells of R agree everywhere; the full R has no unwritten cell.
    mask = region_mask(lx_l, ly_l, N, M, bw).to(cuda)
    assert torch.equal(R0[:, 1:N + 1, 1:M + 1][mask], R1[:, 1:N + 1, 1:M + 1][mask])
    assert not torch.isnan(R0).any()
