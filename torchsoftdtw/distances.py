"""Alias of torchsoftdtw_b200.distances (the reference's module path torchsoftdtw.distances)."""

from torchsoftdtw_b200.distances import (  # noqa: F401
    PAIRWISE_DISTANCES,
    pairwise_cosine,
    pairwise_l1,
    pairwise_l2_squared,
)
