"""Process-group bootstrap and rank helpers.

Public names follow ``abacus/distributed/utils.py`` (``dist_env_vars``,
``init_process_group``, ``shutdown``, ``rank``, ``world_size``,
``print_peak_memory``). The layout is one process per GPU: NCCL bound eagerly
to the process's device on CUDA, gloo over the loopback interface on CPU (the
container hostname need not resolve), one intra-op thread per process so that
co-located CPU ranks do not oversubscribe the cores.
"""
from __future__ import annotations

import datetime
import os
import resource
import sys

import torch
import torch.distributed as dist

_LAUNCHER_KEYS = ("RANK", "WORLD_SIZE")
_LOOPBACK = {"darwin": "lo0"}


def dist_env_vars() -> bool:
    """True when a launcher (torchrun, the test harness) exported the rank layout."""
    return all(key in os.environ for key in _LAUNCHER_KEYS)


def init_process_group(backend: str = "gloo", device: torch.device | None = None,
                       timeout_s: float | None = None) -> None:
    """Join the default process group.

    ``timeout_s`` bounds every collective of the group, so a rank that never
    joins or dies makes the others fail with an error instead of waiting.
    """
    torch.set_num_threads(1)
    options: dict = {"backend": backend}
    if timeout_s is not None:
        options["timeout"] = datetime.timedelta(seconds=timeout_s)
    if backend == "gloo":
        os.environ["GLOO_SOCKET_IFNAME"] = _LOOPBACK.get(sys.platform, "lo")
    else:
        options["device_id"] = device
    dist.init_process_group(**options)


def shutdown() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


def rank() -> int:
    return dist.get_rank()


def world_size() -> int:
    return dist.get_world_size()


def _peak_rss_bytes() -> int:
    # ru_maxrss is in KiB on Linux and in bytes on macOS.
    raw = resource.getrusage(resource.RUSAGE_SELF).ru_maxrss
    return raw if sys.platform == "darwin" else raw * 1024


def print_peak_memory() -> None:
    """Print this process's peak memory: CUDA allocator peak, else host RSS."""
    owner = f"rank {dist.get_rank()}" if dist.is_initialized() else "process"
    if torch.cuda.is_available():
        what, peak = "max CUDA memory", torch.cuda.max_memory_allocated()
    else:
        what, peak = "peak host RSS", _peak_rss_bytes()
    print(f"{owner} {what} {peak / 2**20:.1f} MB", flush=True)
