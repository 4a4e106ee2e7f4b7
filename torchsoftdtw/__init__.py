"""Drop-in import name: ``import torchsoftdtw`` resolves to torchsoftdtw_b200 (same public names as
angelo-ortiz/torchsoftdtw's package), so code written against the reference runs unchanged."""

from torchsoftdtw_b200 import SoftDTW, SoftDTWAutograd, pairwise_cosine, pairwise_l1, pairwise_l2_squared, soft_dtw

from . import distances, softdtw  # noqa: F401

__all__ = [
    "SoftDTW",
    "SoftDTWAutograd",
    "pairwise_cosine",
    "pairwise_l1",
    "pairwise_l2_squared",
    "soft_dtw",
]
