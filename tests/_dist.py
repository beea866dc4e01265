"""Helpers for multi-rank CPU tests: gloo ranks spawned as processes on loopback."""
import os
import socket
import sys
import traceback

import torch.distributed as dist
import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn, args, timeout_s, backend="gloo"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    os.environ["GLOO_SOCKET_IFNAME"] = "lo0" if sys.platform == "darwin" else "lo"
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from abacus_b200.parallel import mesh
    from abacus_b200.utils.dist import init_process_group

    device = None
    if backend == "nccl":
        import torch

        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
    init_process_group(backend, device=device, timeout_s=timeout_s)
    try:
        fn(rank, world, *args)
    except Exception:
        traceback.print_exc()
        raise
    finally:
        mesh.set_mesh(None)
        dist.destroy_process_group()


def run_ranks(fn, world: int, *args, timeout_s: float = 120.0, backend: str = "gloo"):
    """Run fn(rank, world, *args) on `world` ranks (gloo on CPU, or nccl with
    rank r on cuda:r); fails if any rank fails."""
    mp.spawn(_entry, args=(world, free_port(), fn, args, timeout_s, backend), nprocs=world, join=True)
