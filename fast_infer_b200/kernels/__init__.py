"""Attention kernels (drop-in for the reference's ``fast_infer.kernels.attention``)."""

from fast_infer_b200.kernels.attention import flash_attention, paged_attention  # noqa: F401
