"""Tensor-core precision of every abacus_b200 GEMM-shaped kernel.

* ``"fp32"`` (default): 3xTF32 split precision. Each fp32 operand is written
  as hi + lo with both halves exact in tf32, and the tensor core accumulates
  lo*hi + hi*lo + hi*hi in fp32 (Markidis et al. 2018; Ootomo & Yokota 2022).
  The error is at the level of an fp32 SGEMM, which is what the reference
  (true fp32, TF32 disabled) computes.
* ``"tf32"``: one tcgen05 kind::tf32 pass (10-bit mantissa products).
"""
from __future__ import annotations

_PASSES = {"fp32": 3, "tf32": 1}
_precision = "fp32"


def set_precision(mode: str) -> None:
    global _precision
    if mode not in _PASSES:
        raise ValueError(f"precision must be one of {sorted(_PASSES)}, got {mode!r}")
    _precision = mode


def get_precision() -> str:
    return _precision


def passes() -> int:
    return _PASSES[_precision]
