"""Loader for the ``abacus_b200._C`` extension (hand-written sm_100a kernels).

CUDA tensors always run on these kernels: if the extension is missing on a
machine with a GPU, every op raises instead of falling back to ATen. CPU
tensors run the plain PyTorch formulation of the same math (the oracle the
GPU tests compare against, and the path gloo multi-rank tests use).
"""
from __future__ import annotations

import functools

import torch  # noqa: F401  (loads libc10 / libtorch before the extension)


class ExtensionMissing(RuntimeError):
    pass


@functools.lru_cache(maxsize=None)
def ext():
    try:
        from abacus_b200 import _C  # noqa: PLC0415
    except ImportError as error:  # pragma: no cover - depends on the build
        raise ExtensionMissing(
            "abacus_b200._C is not built; run `python setup.py build_ext --inplace` "
            "(CUDA tensors have no fallback path)"
        ) from error
    return _C


def available() -> bool:
    try:
        ext()
    except ExtensionMissing:
        return False
    return True


def check_status(device=None) -> None:
    """Raise if any kernel on `device` recorded a bounded-wait timeout."""
    import torch

    index = torch.cuda.current_device() if device is None else torch.device(device).index or 0
    code = ext().read_status(index)
    if code != 0:
        ext().reset_status(index)
        raise RuntimeError(f"abacus_b200 kernel reported status {code} on cuda:{index}")
