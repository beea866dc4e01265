"""Failure detection on gloo CPU ranks: the failure is made on the host (a
rank reports an error, stops its heartbeat, or never joins a collective) and
the surviving ranks must learn of it within a bounded time."""
import time

import pytest
import torch
import torch.distributed as dist

from _dist import run_ranks
from abacus_b200.utils.fault import Heartbeat, PeerFailure, Watchdog, report_failure


def _reported(rank, world):
    hb = Heartbeat(rank, interval_s=0.1).start()
    dog = Watchdog(world, timeout_s=5.0)
    dist.barrier()
    if rank == 1:
        report_failure("simulated data-loader crash")
        dist.barrier()
        hb.stop()
        return
    dist.barrier()
    with pytest.raises(PeerFailure, match="simulated data-loader crash"):
        dog.check()
    hb.stop()


def test_watchdog_sees_reported_failure():
    run_ranks(_reported, 2)


def _stalled(rank, world):
    hb = Heartbeat(rank, interval_s=0.1).start()
    dog = Watchdog(world, timeout_s=1.0)
    dist.barrier()
    dog.check()  # everyone alive
    if rank == 1:
        hb.stop()  # a hung rank stops beating
        time.sleep(2.5)
        dist.barrier()
        return
    time.sleep(2.0)
    with pytest.raises(PeerFailure, match="rank 1 heartbeat"):
        dog.check()
    hb.stop()
    dist.barrier()


def test_watchdog_sees_stalled_heartbeat():
    run_ranks(_stalled, 2)


def _missing(rank, world):
    if rank == 1:
        time.sleep(6.0)  # never joins the all_reduce below
        return
    start = time.time()
    with pytest.raises(RuntimeError):
        dist.all_reduce(torch.ones(4))
    assert time.time() - start < 30


def test_collective_with_missing_rank_times_out():
    run_ranks(_missing, 2, timeout_s=3.0)
