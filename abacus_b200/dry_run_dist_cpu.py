"""All-reduce sanity check on CPU (gloo) ranks (``scripts/dry_run_dist_cpu.py``).

    torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node=4 -m abacus_b200.dry_run_dist_cpu
"""
import torch
import torch.distributed as dist

from abacus_b200.utils.dist import init_process_group, shutdown


def main() -> None:
    init_process_group("gloo")
    try:
        rank, world = dist.get_rank(), dist.get_world_size()
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t)
        expected = world * (world + 1) / 2
        print(f"rank {rank}/{world}: all_reduce -> {t.item():.0f} (expected {expected:.0f})", flush=True)
        if t.item() != expected:
            raise SystemExit(1)
    finally:
        shutdown()


if __name__ == "__main__":
    main()
