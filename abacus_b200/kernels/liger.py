"""``--liger`` switch at the reference path ``abacus/kernels/liger.py``.

The reference swaps ``F.cross_entropy`` for Liger's Triton kernel when the
flag is set. Here cross entropy always runs on the abacus_b200 CUDA kernel for
CUDA tensors (and the training loop uses the fused linear + cross-entropy
path), so the flag is accepted and recorded but changes nothing.
"""
from __future__ import annotations

from abacus_b200.ops.cross_entropy import cross_entropy  # noqa: F401

_enabled = False


def set_use_liger(enabled: bool) -> None:
    global _enabled
    _enabled = enabled
