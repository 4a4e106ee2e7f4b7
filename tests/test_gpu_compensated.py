"""GPU: the compensated fp32 ops (``torchsoftdtw_b200::forward_x2 / backward_x2``, R kept as R_hi + R_lo) and
``SoftDTW(compensated=True)``, against the oracle in fp64 on the same float32 inputs.

Tolerances: costs rtol 1e-6; R (R_hi + R_lo) rtol 1e-6 / atol 1e-5; E atol 2e-5 * max(1, max|E|) (the default
fp32 path is off by up to 0.07 on the 256 x 512 x 512 gamma = 0.1 workload, the reference's own fp32 backward
by up to 0.67); exact zeros through padding and outside the band.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O
import torchsoftdtw_b200 as T
from torchsoftdtw_b200 import workloads
from test_gpu_ops import PARITY

pytestmark = pytest.mark.gpu


# Same results as the oracle in fp64 on the same float32 D, to a small multiple of float32 rounding, on every
# shape, band and length pattern of the random parity set.
@pytest.mark.parametrize("B,N,M,gamma,bw", PARITY)
def test_compensated_ops_vs_oracle_f64(cuda, B, N, M, gamma, bw):
    rng = np.random.default_rng(B * 31 + N + 7 * M)
    D = (rng.random((B, N, M)) * 3).astype(np.float32)
    lx = rng.integers(max(1, N - 3), N + 1, size=B)
    ly = rng.integers(max(1, M - 3), M + 1, size=B)
    Dd = torch.from_numpy(D).to(cuda)
    lxd, lyd = torch.as_tensor(lx).to(cuda), torch.as_tensor(ly).to(cuda)
    c, Rh, Rl = torch.ops.torchsoftdtw_b200.forward_x2(Dd, lxd, lyd, gamma, bw)
    E = torch.ops.torchsoftdtw_b200.backward_x2(Dd, Rh, Rl, lxd, lyd, gamma, bw)
    torch.cuda.synchronize()
    T.check_errors(cuda)
    c64, R64 = O.forward(D.astype(np.float64), lx, ly, gamma, bw)
    E64 = O.backward(D.astype(np.float64), R64, lx, ly, gamma, bw)
    np.testing.assert_allclose(c.cpu().numpy(), c64, rtol=1e-6, atol=1e-6)
    R = Rh.cpu().numpy().astype(np.float64) + Rl.cpu().numpy().astype(np.float64)
    assert np.array_equal(np.isinf(R), np.isinf(R64))
    fin = np.isfinite(R64)
    np.testing.assert_allclose(R[fin], R64[fin], rtol=1e-6, atol=1e-5)
    En = E.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(En, E64, rtol=0, atol=2e-5 * max(1.0, float(np.max(np.abs(E64)))))
    assert np.all(En[E64 == 0.0] == 0.0)


def test_compensated_module_gradients(cuda):
    """SoftDTW(compensated=True) on the medium workload (16 pairs): float32 gradients closer to the fp64 truth
    than the default path's, and the same costs to fp32 rounding."""
    X, Y, lx, ly, w = workloads.make_inputs("medium", batch=16)
    res = {}
    for comp in (False, True):
        Xd = X.to(cuda).requires_grad_(True)
        c = T.SoftDTW(gamma=w.gamma, compensated=comp)(Xd, Y.to(cuda), lx.to(cuda), ly.to(cuda))
        c.sum().backward()
        torch.cuda.synchronize()
        res[comp] = (c.detach().cpu().numpy(), Xd.grad.cpu().numpy().astype(np.float64))
    c64, gx64, _ = O.module_forward_backward(X.double().numpy(), Y.double().numpy(), lx.numpy(), ly.numpy(),
                                             w.gamma, w.bandwidth, w.normalize)
    np.testing.assert_allclose(res[True][0], c64, rtol=1e-5)
    err_default = np.max(np.abs(res[False][1] - gx64))
    err_comp = np.max(np.abs(res[True][1] - gx64))
    assert err_comp < 0.5 * err_default, (err_comp, err_default)


def test_compensated_rejects_float64(cuda):
    D = torch.rand(2, 5, 5, dtype=torch.float64, device=cuda)
    with pytest.raises(ValueError, match="float32"):
        T.soft_dtw(D, compensated=True)
    with pytest.raises(RuntimeError, match="float32"):
        torch.ops.torchsoftdtw_b200.forward_x2(D, torch.full((2,), 5, device=cuda), torch.full((2,), 5, device=cuda),
                                               1.0, -1)
