"""Alias of torchsoftdtw_b200.softdtw (the reference's module path torchsoftdtw.softdtw)."""

from torchsoftdtw_b200.softdtw import SoftDTW, SoftDTWAutograd, soft_dtw  # noqa: F401
