"""Data-parallel optimizer tail on the benchmark model (~124M fp32 parameters):
NCCL all-reduce of the flat gradient + multi-tensor AdamW, against the fused
peer-memory kernel (barrier with count exchange, reduce + AdamW + broadcast,
barrier). Gradients are random; both paths read inputs far larger than L2.
CUDA events, 5 warm-up and 20 timed iterations, max over ranks.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 benchmarks/bench_ddp_step.py
"""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from abacus_b200.ops._ext import ext  # noqa: E402
from abacus_b200.optim.adamw import AdamW  # noqa: E402
from abacus_b200.parallel.fused_data_parallel import FusedDataParallel  # noqa: E402
from abacus_b200.transformer import Transformer  # noqa: E402


def timed(fn, warmup=5, iters=20):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
    torch.manual_seed(0)
    model = Transformer(dim=768, n_heads=12, head_dim=64, n_blocks=12, vocab_size=50304, hidden_dim=2048).cuda()
    params = list(model.parameters())
    n = sum(p.numel() for p in params)

    # Unfused: one NCCL all-reduce of the flat gradient, scale, AdamW kernel.
    flat = torch.randn(n, device="cuda")
    off = 0
    for p in params:
        p.grad = flat[off : off + p.numel()].view_as(p)
        off += p.numel()
    opt = AdamW(model)

    def unfused():
        dist.all_reduce(flat)
        flat.mul_(1.0 / world)
        opt.step()

    t_unfused = timed(unfused)

    # Fused: gradients already in the symmetric buffer (the hooks' copy is
    # part of backward in both paths).
    fused_model = Transformer(dim=768, n_heads=12, head_dim=64, n_blocks=12, vocab_size=50304,
                              hidden_dim=2048).cuda()
    dp = FusedDataParallel(fused_model, overlap=False)
    dp.broadcast_parameters()
    fopt = AdamW(fused_model, owned=dp.owned)
    dp.bind_optimizer(fopt)
    dp._grad_flat.normal_()
    loss = torch.ones((), device="cuda")
    count = torch.tensor(1000, device="cuda")

    def fused():
        dp.prepare_step(fopt, count)
        for b in dp.flat_buckets:
            b.arrived.update(b.members)
        dp.synchronize(loss, count)

    t_fused = timed(fused)
    dp.check()
    nbytes = 4 * n
    if rank == 0:
        print(json.dumps({
            "world": world, "params": n,
            "unfused_ms": round(t_unfused, 3), "fused_ms": round(t_fused, 3),
            "fused_nvlink_gbs_per_rank": round(2 * nbytes * (world - 1) / world / t_fused / 1e6, 1),
            "launches": ext().launch_count(),
        }), flush=True)
    torch.cuda.synchronize()
    dp.release()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
