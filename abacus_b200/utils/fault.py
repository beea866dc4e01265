"""Failure detection for multi-rank training, without faulting a GPU.

* ``Heartbeat``: a daemon thread that writes this rank's wall-clock time to
  the process group's key-value store every ``interval_s``.
* ``Watchdog``: ``check()`` raises ``PeerFailure`` when a peer reported a
  failure (``report_failure``) or its heartbeat is older than ``timeout_s``.
  Call it between steps, before the next collective is launched, so a dead or
  hung rank ends the others' step with an exception instead of a collective
  that waits forever.
* ``check_device()``: raises if an abacus kernel on this GPU recorded a
  bounded-wait timeout (a peer flag that never arrived, a stalled pipeline)
  in the device status word; the context itself stays usable.

The reference framework has no failure detection (an exception on one rank
leaves the others blocked in NCCL).
"""
from __future__ import annotations

import threading
import time

import torch.distributed as dist


class PeerFailure(RuntimeError):
    pass


def _store(store=None):
    if store is not None:
        return store
    from torch.distributed import distributed_c10d

    return distributed_c10d._get_default_store()


class Heartbeat:
    def __init__(self, rank: int, interval_s: float = 0.5, store=None, prefix: str = "abacus/hb"):
        self.rank = rank
        self.interval_s = interval_s
        self.store = _store(store)
        self.prefix = prefix
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def beat(self) -> None:
        self.store.set(f"{self.prefix}/{self.rank}", repr(time.time()))

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self.beat()
            except Exception:  # noqa: BLE001 - the store went away: stop beating
                return
            self._stop.wait(self.interval_s)

    def start(self) -> "Heartbeat":
        self.beat()
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=5)


def report_failure(message: str, rank: int | None = None, store=None, prefix: str = "abacus/fail") -> None:
    """Publish a failure so every peer's Watchdog.check() raises."""
    rank = dist.get_rank() if rank is None else rank
    _store(store).set(f"{prefix}/{rank}", message)


class Watchdog:
    def __init__(self, world_size: int, timeout_s: float = 10.0, store=None, hb_prefix: str = "abacus/hb",
                 fail_prefix: str = "abacus/fail"):
        self.world_size = world_size
        self.timeout_s = timeout_s
        self.store = _store(store)
        self.hb_prefix = hb_prefix
        self.fail_prefix = fail_prefix

    def check(self) -> None:
        now = time.time()
        fail_keys = [f"{self.fail_prefix}/{r}" for r in range(self.world_size)]
        for r, key in enumerate(fail_keys):
            if self.store.check([key]):
                raise PeerFailure(f"rank {r} reported a failure: {self.store.get(key).decode()}")
        for r in range(self.world_size):
            key = f"{self.hb_prefix}/{r}"
            if not self.store.check([key]):
                raise PeerFailure(f"rank {r} has no heartbeat")
            last = float(self.store.get(key).decode())
            if now - last > self.timeout_s:
                raise PeerFailure(f"rank {r} heartbeat is {now - last:.1f} s old")


def check_device(device=None) -> None:
    """Raise if an abacus kernel recorded an error status on this device."""
    from abacus_b200.ops._ext import check_status

    check_status(device)
