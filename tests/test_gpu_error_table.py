"""GPU: the fp32 gradient error table. For each workload (the sizes the oracle finishes in seconds), the max
error of this library's fp32 results against the oracle in fp64 on the same inputs, next to the reference's
own fp32 error (the oracle in fp32, bit-identical to the reference's CPU operator):

* module level: costs (relative) and grad_X of ``SoftDTW(...)(X, Y).sum()`` (X, Y float32 -> fp64 truth from the
  same float32 inputs);
* op level: E = d costs / d D on the same float32 D, by the default ops and by the compensated ops
  (``torchsoftdtw_b200::forward_x2 / backward_x2``, R kept as R_hi + R_lo).

Run with ``-s`` to print the table (one JSON line per workload). The assertions pin the ratios: this library's
gradient error is at most 0.25 times the reference's on every workload (measured 0.02-0.13), and the
compensated ops' E error at most 0.01 times the reference's.
"""

import json

import numpy as np
import pytest
import torch

from oracle import oracle as O
import torchsoftdtw_b200 as T
from torchsoftdtw_b200 import workloads

pytestmark = pytest.mark.gpu

RATIO = 0.25


@pytest.mark.parametrize("name,batch", [("readme", 8), ("medium", 16), ("ragged", 128), ("long", 1)])
def test_fp32_gradient_error_table(cuda, name, batch):
    X, Y, lx, ly, w = workloads.make_inputs(name, batch=batch)
    Xn, Yn, lxn, lyn = X.numpy(), Y.numpy(), lx.numpy(), ly.numpy()
    Xd = X.to(cuda).requires_grad_(True)
    c = T.SoftDTW(gamma=w.gamma, bandwidth=w.bandwidth, normalize=w.normalize)(Xd, Y.to(cuda), lx.to(cuda),
                                                                                ly.to(cuda))
    c.sum().backward()
    torch.cuda.synchronize()
    T.check_errors(cuda)
    gx = Xd.grad.cpu().numpy().astype(np.float64)
    c64, gx64, _ = O.module_forward_backward(Xn.astype(np.float64), Yn.astype(np.float64), lxn, lyn, w.gamma,
                                             w.bandwidth, w.normalize)
    c32, gx32, _ = O.module_forward_backward(Xn, Yn, lxn, lyn, w.gamma, w.bandwidth, w.normalize)
    D32 = O.pairwise_l2_squared(Xn, Yn)[0].astype(np.float32)
    Dd = torch.from_numpy(D32).to(cuda)
    _, R = torch.ops.torchsoftdtw.forward(Dd, lx.to(cuda), ly.to(cuda), w.gamma, w.bandwidth)
    E = torch.ops.torchsoftdtw.backward(Dd, R, lx.to(cuda), ly.to(cuda), w.gamma, w.bandwidth)
    E = E.cpu().numpy().astype(np.float64)
    _, R64 = O.forward(D32.astype(np.float64), lxn, lyn, w.gamma, w.bandwidth)
    E64 = O.backward(D32.astype(np.float64), R64, lxn, lyn, w.gamma, w.bandwidth)
    _, R32 = O.forward(D32, lxn, lyn, w.gamma, w.bandwidth)
    E32 = O.backward(D32, R32, lxn, lyn, w.gamma, w.bandwidth).astype(np.float64)
    cx, Rh, Rl = torch.ops.torchsoftdtw_b200.forward_x2(Dd, lx.to(cuda), ly.to(cuda), w.gamma, w.bandwidth)
    Ex = torch.ops.torchsoftdtw_b200.backward_x2(Dd, Rh, Rl, lx.to(cuda), ly.to(cuda), w.gamma, w.bandwidth)
    torch.cuda.synchronize()
    T.check_errors(cuda)
    Ex = Ex.cpu().numpy().astype(np.float64)
    c64op, _ = O.forward(D32.astype(np.float64), lxn, lyn, w.gamma, w.bandwidth)
    with np.errstate(invalid="ignore"):
        row = {
            "workload": name, "batch": batch, "gamma": w.gamma,
            "cost_rel_ours": float(np.max(np.abs(c.detach().cpu().numpy() - c64) / np.abs(c64))),
            "cost_rel_ref": float(np.max(np.abs(c32 - c64) / np.abs(c64))),
            "grad_x_abs_ours": float(np.max(np.abs(gx - gx64))),
            "grad_x_abs_ref": float(np.nanmax(np.abs(gx32 - gx64))),
            "grad_x_max": float(np.max(np.abs(gx64))),
            "E_abs_ours": float(np.max(np.abs(E - E64))),
            "E_abs_ref": float(np.nanmax(np.abs(E32 - E64))),
            "E_abs_compensated": float(np.max(np.abs(Ex - E64))),
            "cost_rel_compensated": float(np.max(np.abs(cx.cpu().numpy() - c64op) / np.abs(c64op))),
        }
    print(json.dumps(row))
    assert row["cost_rel_ours"] <= 1e-5
    assert row["grad_x_abs_ours"] <= RATIO * row["grad_x_abs_ref"], row
    assert row["E_abs_ours"] <= RATIO * row["E_abs_ref"], row
    assert row["E_abs_compensated"] <= 0.01 * row["E_abs_ref"], row
    assert row["cost_rel_compensated"] <= 1e-6, row
    # exact zeros through padding and outside the band, as on the default path
    assert np.all(Ex[E64 == 0.0] == 0.0)
