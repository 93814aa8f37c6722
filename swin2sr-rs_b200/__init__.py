"""swin2sr-rs_b200: a B200-native Swin2SR forward pass behind the reference's Backend API.

The package mirrors the reference's host interface for the one hot path it
accelerates (``src/backend.rs`` ``Backend`` trait, ``src/plan.rs``,
``src/weights.rs``). The arithmetic lives in ``csrc/`` (sm_100a CUDA kernels
behind the C ABI of ``include/s2s.h``), loaded through ``capi``.
"""
from . import plan, weights  # noqa: F401

__all__ = ["plan", "weights"]
