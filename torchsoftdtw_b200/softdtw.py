"""Soft-DTW operator and module, a drop-in for the reference's ``src/torchsoftdtw/softdtw.py``.

Same public names, signatures, defaults, errors and numerics contract:

* ``torch.ops.torchsoftdtw.forward(D, lengths_x, lengths_y, gamma, bandwidth) -> (costs, R)`` and
  ``torch.ops.torchsoftdtw.backward(D, R, lengths_x, lengths_y, gamma, bandwidth) -> E`` with the
  reference's schemas (``softdtw.cpp:342-345``) and FakeTensor kernels (``softdtw.py:18-30``);
* :class:`SoftDTWAutograd` and :func:`soft_dtw` (``softdtw.py:33-77``);
* :class:`SoftDTW` (``softdtw.py:80-142``), whose ``l2_squared`` path on CUDA runs this library's fused
  ops ``torchsoftdtw_b200::l2_forward`` / ``l2_backward`` (cost matrix, wavefront and the gradient
  contraction in native kernels) instead of building D with tensor expressions.

Everything runs on CUDA (sm_100); CPU tensors are validated like the reference's and then rejected.
"""

import torch
from torch import nn
from torch.autograd import Function

from . import _ext
from .distances import PAIRWISE_DISTANCES

_ext.load()


def _acc_dtype(dtype: torch.dtype) -> torch.dtype:
    if dtype in (torch.float16, torch.bfloat16):
        return torch.float32
    return dtype


# ---- FakeTensor kernels for torch.compile ----


@torch.library.register_fake("torchsoftdtw::forward")
def _forward_fake(D, lengths_x, lengths_y, gamma, bandwidth):
    B, N, M = D.shape
    acc_dt = _acc_dtype(D.dtype)
    costs = D.new_empty((B,), dtype=acc_dt)
    R = D.new_empty((B, N + 2, M + 2), dtype=acc_dt)
    return costs, R


@torch.library.register_fake("torchsoftdtw::backward")
def _backward_fake(D, R, lengths_x, lengths_y, gamma, bandwidth):
    B, N, M = D.shape
    return D.new_empty((B, N, M))


@torch.library.register_fake("torchsoftdtw_b200::l2_forward")
def _l2_forward_fake(X, Y, lengths_x, lengths_y, gamma, bandwidth):
    B, N, _ = X.shape
    M = Y.shape[1]
    acc_dt = _acc_dtype(X.dtype)
    # R is the forward's strip tiles when the pair-resident kernels run both directions (a property of the
    # shape, the dtype and the device, asked of the library), else the padded R.
    if _ext.r_tiled(int(B), int(N), int(M), acc_dt, X.device):
        R = X.new_empty((B, (N + 31) // 32, (M + 31) // 32 + 1, 32, 32), dtype=acc_dt)
    else:
        R = X.new_empty((B, N + 2, M + 2), dtype=acc_dt)
    if _ext.l2_fused(int(B), int(N), int(M), int(X.shape[2]), acc_dt, X.device):
        # The cost matrix stays inside the forward: the third output is its clamp mask (one bit per cell).
        Dout = X.new_empty((B, N, (M + 31) // 32), dtype=torch.int32)
    else:
        Dout = X.new_empty((B, N, M), dtype=acc_dt)
    return (X.new_empty((B,), dtype=acc_dt), R, Dout, X.new_empty((B,), dtype=torch.int32))


@torch.library.register_fake("torchsoftdtw_b200::forward_x2")
def _forward_x2_fake(D, lengths_x, lengths_y, gamma, bandwidth):
    B, N, M = D.shape
    f32 = torch.float32
    return (D.new_empty((B,), dtype=f32), D.new_empty((B, N + 2, M + 2), dtype=f32),
            D.new_empty((B, N + 2, M + 2), dtype=f32))


@torch.library.register_fake("torchsoftdtw_b200::backward_x2")
def _backward_x2_fake(D, R_hi, R_lo, lengths_x, lengths_y, gamma, bandwidth):
    B, N, M = D.shape
    return D.new_empty((B, N, M))


@torch.library.register_fake("torchsoftdtw_b200::l2_backward")
def _l2_backward_fake(X, Y, D, R, clamp_flags, lengths_x, lengths_y, grad_costs, gamma, bandwidth, need_x, need_y):
    gX = X.new_empty(X.shape) if need_x else X.new_empty((0,))
    gY = Y.new_empty(Y.shape) if need_y else Y.new_empty((0,))
    return gX, gY


@torch.library.register_fake("torchsoftdtw_b200::dist_forward")
def _dist_forward_fake(X, Y, lengths_x, lengths_y, gamma, bandwidth, kind, eps):
    B, N, M = X.shape[0], X.shape[1], Y.shape[1]
    acc = _acc_dtype(X.dtype)
    return (X.new_empty((B,), dtype=acc), X.new_empty((B, N + 2, M + 2), dtype=acc),
            X.new_empty((B, N, M), dtype=acc))


@torch.library.register_fake("torchsoftdtw_b200::dist_backward")
def _dist_backward_fake(X, Y, D, R, lengths_x, lengths_y, grad_costs, gamma, bandwidth, kind, eps, need_x, need_y):
    gX = X.new_empty(X.shape) if need_x else X.new_empty((0,))
    gY = Y.new_empty(Y.shape) if need_y else Y.new_empty((0,))
    return gX, gY


class SoftDTWAutograd(Function):
    """Autograd of the op pair (``softdtw.py:33-48``): saves D and R, returns grad_output * E."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, D, lengths_x, lengths_y, gamma, bandwidth):
        costs, R = torch.ops.torchsoftdtw.forward(D, lengths_x, lengths_y, gamma, bandwidth)
        ctx.save_for_backward(D, R, lengths_x, lengths_y)
        ctx.gamma = gamma
        ctx.bandwidth = bandwidth
        return costs

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_output):
        D, R, lengths_x, lengths_y = ctx.saved_tensors
        E = torch.ops.torchsoftdtw.backward(D, R, lengths_x, lengths_y, ctx.gamma, ctx.bandwidth)
        return grad_output.unsqueeze(-1).unsqueeze(-1) * E, None, None, None, None


class _SoftDTWCompensated(Function):
    """SoftDTWAutograd over the compensated fp32 ops (R kept as R_hi + R_lo): the better-conditioned fp32
    backward. Costs in float32, the gradient in D's dtype."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, D, lengths_x, lengths_y, gamma, bandwidth):
        costs, R_hi, R_lo = torch.ops.torchsoftdtw_b200.forward_x2(D, lengths_x, lengths_y, gamma, bandwidth)
        ctx.save_for_backward(D, R_hi, R_lo, lengths_x, lengths_y)
        ctx.gamma = gamma
        ctx.bandwidth = bandwidth
        return costs

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_output):
        D, R_hi, R_lo, lengths_x, lengths_y = ctx.saved_tensors
        E = torch.ops.torchsoftdtw_b200.backward_x2(D, R_hi, R_lo, lengths_x, lengths_y, ctx.gamma, ctx.bandwidth)
        return grad_output.unsqueeze(-1).unsqueeze(-1).to(E.dtype) * E, None, None, None, None


class _SoftDTWL2(Function):
    """Fused squared-L2 path: costs from (X, Y) and gradients w.r.t. X and Y, all in native kernels.

    Mathematically the composition pairwise_l2_squared -> SoftDTWAutograd (including the clamp's
    zero gradient where |x|^2 + |y|^2 - 2 x.y < 0), without materialising grad_output * E."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, X, Y, lengths_x, lengths_y, gamma, bandwidth):
        costs, R, D, flags = torch.ops.torchsoftdtw_b200.l2_forward(X, Y, lengths_x, lengths_y, gamma, bandwidth)
        ctx.save_for_backward(X, Y, D, R, flags, lengths_x, lengths_y)
        ctx.gamma = gamma
        ctx.bandwidth = bandwidth
        return costs

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_costs):
        X, Y, D, R, flags, lengths_x, lengths_y = ctx.saved_tensors
        need_x, need_y = bool(ctx.needs_input_grad[0]), bool(ctx.needs_input_grad[1])
        gX, gY = torch.ops.torchsoftdtw_b200.l2_backward(
            X, Y, D, R, flags, lengths_x, lengths_y, grad_costs.contiguous(), ctx.gamma, ctx.bandwidth, need_x, need_y
        )
        return (gX if need_x else None), (gY if need_y else None), None, None, None, None


# distance name -> kind code of the native L1 / cosine cost kernels
_DIST_KIND = {"l1": 1, "cosine": 2}
_COSINE_EPS = 1e-8  # pairwise_cosine's default floor of the norms (distances.py:34)


class _SoftDTWDist(Function):
    """L1 / cosine path: the cost matrix from (X, Y) in native kernels, the Soft-DTW ops, and the gradient
    w.r.t. X and Y contracted in native kernels (no (B, N, M, d) difference tensor, no grad_output * E).
    Mathematically the composition pairwise_l1 / pairwise_cosine -> SoftDTWAutograd."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, X, Y, lengths_x, lengths_y, gamma, bandwidth, kind, eps):
        costs, R, D = torch.ops.torchsoftdtw_b200.dist_forward(X, Y, lengths_x, lengths_y, gamma, bandwidth, kind,
                                                               eps)
        ctx.save_for_backward(X, Y, D, R, lengths_x, lengths_y)
        ctx.gamma, ctx.bandwidth, ctx.kind, ctx.eps = gamma, bandwidth, kind, eps
        return costs

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_costs):
        X, Y, D, R, lengths_x, lengths_y = ctx.saved_tensors
        need_x, need_y = bool(ctx.needs_input_grad[0]), bool(ctx.needs_input_grad[1])
        gX, gY = torch.ops.torchsoftdtw_b200.dist_backward(
            X, Y, D, R, lengths_x, lengths_y, grad_costs.contiguous(), ctx.gamma, ctx.bandwidth, ctx.kind, ctx.eps,
            need_x, need_y)
        return (gX if need_x else None), (gY if need_y else None), None, None, None, None, None, None


def soft_dtw(
    D: torch.Tensor,
    lengths_x: torch.Tensor | None = None,
    lengths_y: torch.Tensor | None = None,
    gamma: float = 1.0,
    bandwidth: int = -1,
    dp_dtype: torch.dtype | None = None,
    compensated: bool = False,
) -> torch.Tensor:
    """Compute soft-DTW on a pre-computed cost matrix.

    Args:
        D: (B, N, M) pairwise cost matrix.
        lengths_x: (B,) actual lengths along dim 1, int32 or int64. Defaults to N for all.
        lengths_y: (B,) actual lengths along dim 2, int32 or int64. Defaults to M for all.
        gamma: Smoothing parameter (> 0).
        bandwidth: Sakoe-Chiba bandwidth around the diagonal joining (0, 0) to (lengths_x - 1, lengths_y - 1),
            in steps along the longer axis. Floored at half the diagonal's slope so that a warping path always
            exists. -1 means no constraint.
        dp_dtype: dtype the dynamic program runs in (None: D's accumulation dtype, as in the reference).
            ``torch.float64`` for a float32 D is the better-conditioned option: the backward's softmin
            weights come from differences of neighbouring R values, which in float32 carry an absolute
            error of about ulp(R) and, divided by a small gamma, make float32 gradients noisy; in float64
            they do not. Costs and gradients are returned in D's dtype. An addition of this package (the
            reference has no such argument); the default leaves the reference's behaviour unchanged.
        compensated: for a float32 (or float16 / bfloat16) D, run the dynamic program in compensated float32:
            R kept as the unevaluated sum of two floats, so the backward's softmin weights come from R
            differences accurate far below ulp(R). Better-conditioned fp32 gradients without float64
            arithmetic (float32 costs, the gradient in D's dtype); slower than the default kernels. An addition
            of this package.

    Returns:
        costs: (B,) soft-DTW values.
    """
    B, N, M = D.shape
    if lengths_x is None:
        lengths_x = torch.full((B,), N, dtype=torch.long, device=D.device)
    if lengths_y is None:
        lengths_y = torch.full((B,), M, dtype=torch.long, device=D.device)
    if compensated:
        if D.dtype == torch.float64:
            raise ValueError("compensated=True is a float32 option; float64 D needs no compensation")
        return _SoftDTWCompensated.apply(D, lengths_x, lengths_y, gamma, bandwidth)
    if dp_dtype is not None and dp_dtype != D.dtype:
        return SoftDTWAutograd.apply(D.to(dp_dtype), lengths_x, lengths_y, gamma, bandwidth).to(D.dtype)
    return SoftDTWAutograd.apply(D, lengths_x, lengths_y, gamma, bandwidth)


class SoftDTW(nn.Module):
    def __init__(
        self,
        gamma: float = 1.0,
        bandwidth: int = -1,
        normalize: bool = False,
        distance: str = "l2_squared",
        dp_dtype: torch.dtype | None = None,
        compensated: bool = False,
    ):
        """
        Args:
            gamma: Smoothing parameter (> 0).
            bandwidth: Sakoe-Chiba bandwidth around the diagonal joining the first and last frames, in steps
                along the longer sequence. Floored at half the diagonal's slope so that a warping path always
                exists. -1 means no constraint.
            normalize: Divide the cost by path length (lengths_x + lengths_y - 1).
            distance: Pairwise distance used to build the cost matrix from X, Y.
                One of "l2_squared", "l1", "cosine".
            dp_dtype: dtype of the computation (None: the inputs' accumulation dtype, as in the reference).
                ``torch.float64`` with float32 inputs is the better-conditioned option (see ``soft_dtw``):
                the cost matrix and the dynamic program run in float64 and the costs and gradients come back
                in the inputs' dtype. Not an argument of the reference; the default keeps its behaviour.
            compensated: float32 inputs only: the dynamic program in compensated float32 (see ``soft_dtw``), the
                better-conditioned fp32 backward. The cost matrix is the distance's tensor expression and its
                gradient flows through torch autograd. Not an argument of the reference.
        """
        super().__init__()
        if distance not in PAIRWISE_DISTANCES:
            raise ValueError(f"Unknown distance {distance!r}, expected one of {sorted(PAIRWISE_DISTANCES)}")
        self.gamma = gamma
        self.bandwidth = bandwidth
        self.normalize = normalize
        self.distance = distance
        self.dp_dtype = dp_dtype
        self.compensated = compensated

    def forward(
        self,
        X: torch.Tensor,
        Y: torch.Tensor,
        lengths_x: torch.Tensor | None = None,
        lengths_y: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Compute soft-DTW between sequences X and Y.

        Args:
            X: (B, N, D) or (N, D) input sequences.
            Y: (B, M, D) or (M, D) target sequences.
            lengths_x: (B,) actual sequence lengths for X.
            lengths_y: (B,) actual sequence lengths for Y.

        Returns:
            costs: (B,) soft-DTW distances.
        """
        if X.dim() == 2:
            X = X.unsqueeze(0)
        if Y.dim() == 2:
            Y = Y.unsqueeze(0)
        out_dtype = None
        if self.dp_dtype is not None and (X.dtype != self.dp_dtype or Y.dtype != self.dp_dtype):
            out_dtype = torch.promote_types(X.dtype, Y.dtype)
            X, Y = X.to(self.dp_dtype), Y.to(self.dp_dtype)

        B = X.size(0)

        if self.compensated:
            D = PAIRWISE_DISTANCES[self.distance](X, Y)
            costs = soft_dtw(D, lengths_x, lengths_y, self.gamma, self.bandwidth, compensated=True)
        elif X.is_cuda and Y.is_cuda and X.dtype == Y.dtype:
            lx = lengths_x if lengths_x is not None else torch.full((B,), X.size(1), dtype=torch.long, device=X.device)
            ly = lengths_y if lengths_y is not None else torch.full((B,), Y.size(1), dtype=torch.long, device=X.device)
            if self.distance == "l2_squared":
                costs = _SoftDTWL2.apply(X, Y, lx, ly, self.gamma, self.bandwidth)
            else:
                costs = _SoftDTWDist.apply(X, Y, lx, ly, self.gamma, self.bandwidth, _DIST_KIND[self.distance],
                                           _COSINE_EPS)
        else:
            D = PAIRWISE_DISTANCES[self.distance](X, Y)
            costs = soft_dtw(D, lengths_x, lengths_y, self.gamma, self.bandwidth)

        if self.normalize:
            if lengths_x is None:
                lengths_x = torch.full((B,), X.size(1), dtype=torch.long, device=X.device)
            if lengths_y is None:
                lengths_y = torch.full((B,), Y.size(1), dtype=torch.long, device=Y.device)
            costs = costs / (lengths_x + lengths_y - 1).to(costs.dtype)
        return costs if out_dtype is None else costs.to(out_dtype)
