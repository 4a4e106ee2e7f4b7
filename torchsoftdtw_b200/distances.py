"""Pairwise cost functions, with the reference's names and semantics
(``src/torchsoftdtw/distances.py:4-57``).

These are differentiable tensor expressions usable on any device. On CUDA the ``SoftDTW`` module does
not call them: it computes the cost matrix, the wavefront and the gradient contraction in this library's
kernels (``torchsoftdtw_b200::l2_forward`` / ``l2_backward`` for ``l2_squared``, ``dist_forward`` /
``dist_backward`` for ``l1`` and ``cosine``, with the same eps = 1e-8 floor of the cosine norms).
"""

import torch


def pairwise_l2_squared(X: torch.Tensor, Y: torch.Tensor) -> torch.Tensor:
    """D[b,i,j] = ||X[b,i] - Y[b,j]||^2 = |x|^2 + |y|^2 - 2 x.y, clamped at 0 (distances.py:4-18).

    Args:
        X: (B, N, D)
        Y: (B, M, D)
    Returns:
        D: (B, N, M)
    """
    x2 = (X * X).sum(dim=-1)
    y2 = (Y * Y).sum(dim=-1)
    xy = torch.bmm(X, Y.transpose(1, 2))
    D = x2.unsqueeze(2) + y2.unsqueeze(1) - 2 * xy
    return D.clamp_min(0.0)


def pairwise_l1(X: torch.Tensor, Y: torch.Tensor) -> torch.Tensor:
    """D[b,i,j] = sum_d |X[b,i,d] - Y[b,j,d]| (distances.py:21-31)."""
    return (X.unsqueeze(2) - Y.unsqueeze(1)).abs().sum(dim=-1)


def pairwise_cosine(X: torch.Tensor, Y: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    """D[b,i,j] = 1 - cos_sim(X[b,i], Y[b,j]), norms floored at eps (distances.py:34-50)."""
    x_norm = X.norm(dim=-1, keepdim=True).clamp_min(eps)
    y_norm = Y.norm(dim=-1, keepdim=True).clamp_min(eps)
    sim = torch.bmm(X / x_norm, (Y / y_norm).transpose(1, 2))
    return 1.0 - sim


PAIRWISE_DISTANCES = {
    "l2_squared": pairwise_l2_squared,
    "l1": pairwise_l1,
    "cosine": pairwise_cosine,
}
