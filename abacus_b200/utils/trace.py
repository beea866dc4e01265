"""Per-phase tracing of a training step: NVTX ranges and device times.

The reference has no tracing (its examples print wall-clock time only). Here
every phase of ``Trainer.step`` (``forward``, ``backward``, ``dp_sync``,
``optimizer``, and the pipeline / context-parallel variants) runs inside
``PhaseTracer.phase``:

* an NVTX range named ``abacus/<phase>`` (visible in Nsight Systems / Nsight
  Compute range filters), pushed on the host when the phase's work is issued;
* optionally (``timing=True``) a pair of CUDA events on the current stream, so
  ``times_ms()`` returns the device time of each phase summed since the last
  call. On CPU the host clock is used instead.

NVTX is on by default when CUDA is available (a range costs about a
microsecond of host time); set ``ABACUS_NVTX=0`` to switch it off.
"""
from __future__ import annotations

import contextlib
import os
import time
from collections import defaultdict

import torch


def _nvtx_default() -> bool:
    return torch.cuda.is_available() and os.environ.get("ABACUS_NVTX", "1") != "0"


class PhaseTracer:
    def __init__(self, nvtx: bool | None = None, timing: bool = False):
        self.nvtx = _nvtx_default() if nvtx is None else bool(nvtx and torch.cuda.is_available())
        self.timing = timing
        self._pending: list[tuple[str, object, object]] = []
        self._host: dict[str, float] = defaultdict(float)

    @contextlib.contextmanager
    def phase(self, name: str, device: torch.device | None = None):
        on_gpu = self.timing and torch.cuda.is_available() and (device is None or device.type == "cuda")
        if self.nvtx:
            torch.cuda.nvtx.range_push(f"abacus/{name}")
        start = end = None
        if on_gpu:
            start = torch.cuda.Event(enable_timing=True)
            start.record()
        elif self.timing:
            t0 = time.perf_counter()
        try:
            yield
        finally:
            if on_gpu:
                end = torch.cuda.Event(enable_timing=True)
                end.record()
                self._pending.append((name, start, end))
            elif self.timing:
                self._host[name] += (time.perf_counter() - t0) * 1e3
            if self.nvtx:
                torch.cuda.nvtx.range_pop()

    def times_ms(self) -> dict[str, float]:
        """Time per phase (ms) since the last call (device time on CUDA)."""
        out: dict[str, float] = defaultdict(float)
        for name, start, end in self._pending:
            end.synchronize()
            out[name] += start.elapsed_time(end)
        for name, ms in self._host.items():
            out[name] += ms
        self._pending.clear()
        self._host.clear()
        return dict(out)
