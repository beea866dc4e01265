"""the CPU / gloo world-size-2 data-parallel plumbing run.

Model: 4 layers, d_model 256, 4 heads x 64, SwiGLU hidden 688, RoPE, QK-norm,
vocab 50304, fp32, random init. Data: seq_len 256, per-rank batch 4,
uniform-random int64 tokens from seed 0 (257 tokens per row, so 256 targets).
AdamW lr 3e-4, betas (0.9, 0.95), weight decay 0.1 under WSD, 20 steps.
Throughput is counted over steps 6-20 (host clock around ``Trainer.step``,
which ends in a host read of the loss), max over the two ranks.

    python benchmarks/bench_cpu_config1.py [--impl abacus|reference|both] [--stages 0 1 2 3]

``--impl reference`` runs the reference from ``baseline/_ref`` through its own
``Transformer`` / ``DataParallel`` / ``Trainer``, with ``abacus.mlp.MLP(256,
688)`` assigned to each block (the reference hard-codes a 4 * dim hidden
size). Its ZeRO stages call ``dist.all_gather_single`` /
``reduce_scatter_single``, which torch 2.11 lacks; for those stages the two
names are bound to ``all_gather_into_tensor`` / ``reduce_scatter_tensor``
(same semantics) in this process, without touching the reference's files.
"""
import argparse
import json
import os
import socket
import sys
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MODEL = dict(dim=256, n_heads=4, head_dim=64, n_blocks=4, vocab_size=50304)
HIDDEN = 688
SEQ, BATCH, STEPS, SKIP = 256, 4, 20, 5


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _build(impl, stage):
    if impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        if not hasattr(dist, "all_gather_single"):
            dist.all_gather_single = dist.all_gather_into_tensor
        if not hasattr(dist, "reduce_scatter_single"):
            dist.reduce_scatter_single = dist.reduce_scatter_tensor
        from abacus.distributed.data_parallel import DataParallel
        from abacus.mlp import MLP
        from abacus.trainer import Trainer
        from abacus.transformer import Transformer

        torch.manual_seed(0)
        model = Transformer(**MODEL)
        for block in model.blocks:
            block.mlp = MLP(MODEL["dim"], HIDDEN)
        trainer = Trainer(model, DataParallel(model, stage=stage), total_steps=STEPS)
    else:
        sys.path.insert(0, ROOT)
        from abacus_b200.distributed.data_parallel import DataParallel
        from abacus_b200.trainer import Trainer
        from abacus_b200.transformer import Transformer

        torch.manual_seed(0)
        model = Transformer(**MODEL, hidden_dim=HIDDEN)
        trainer = Trainer(model, DataParallel(model, stage=stage), total_steps=STEPS, device="cpu")
    # AdamW betas / weight decay of the config; the WSD peak learning rate 3e-4
    # (both trainers build AdamW and WSD themselves; these are their fields).
    opt = trainer.optimizer
    opt.beta1, opt.beta2, opt.weight_decay = 0.9, 0.95, 0.1
    trainer.scheduler.lr = 3e-4
    opt.lr = trainer.scheduler.learning_rate(1)
    return trainer


def _rank(rank, world, port, impl, stage, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      GLOO_SOCKET_IFNAME="lo")
    torch.set_num_threads(1)
    dist.init_process_group("gloo")
    try:
        trainer = _build(impl, stage)
        gen = torch.Generator().manual_seed(0 + 1_000_003 * rank)
        batches = [torch.randint(0, MODEL["vocab_size"], (BATCH, SEQ + 1), generator=gen) for _ in range(STEPS)]
        elapsed = 0.0
        for i, tokens in enumerate(batches):
            t0 = time.perf_counter()
            loss, _ = trainer.step(tokens)
            float(loss)
            if i >= SKIP:
                elapsed += time.perf_counter() - t0
        t = torch.tensor([elapsed], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            tokens_counted = world * BATCH * SEQ * (STEPS - SKIP)
            out.put({"impl": impl, "stage": stage, "tokens_per_s": tokens_counted / float(t), "loss": float(loss)})
    finally:
        dist.destroy_process_group()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--impl", choices=("abacus", "reference", "both"), default="both")
    p.add_argument("--stages", type=int, nargs="+", default=[0, 1, 2, 3])
    args = p.parse_args()
    impls = ["reference", "abacus"] if args.impl == "both" else [args.impl]
    ctx = mp.get_context("spawn")
    for impl in impls:
        if impl == "reference" and not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "abacus")):
            print(json.dumps({"impl": impl, "unavailable": "reference not installed in baseline/_ref"}))
            continue
        for stage in args.stages:
            q = ctx.Queue()
            mp.start_processes(_rank, args=(2, _port(), impl, stage, q), nprocs=2, join=True, start_method="spawn")
            print(json.dumps(q.get()), flush=True)


if __name__ == "__main__":
    main()
