"""Training throughput of the other benchmark configurations, both arms.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/bench_configs.py \\
        --config {tp,moe,cppp} [--impl abacus|reference] [--steps K] [--warmup W]

Configs (synthetic uniform-random int64 tokens, seed 0; random-init weights;
fp32 parameters; timing as in bench.py: W untimed steps, then exactly K steps
between barrier + synchronize, CUDA events, max over ranks; one JSON line):

* ``tp``: ~1.3B dense GPT, 24 layers, d_model 2048, 16 heads x 128, SwiGLU
  5632, vocab 50304, seq_len 2048, global batch 16, tensor parallel TP=N with
  Megatron sequence parallel (every TP rank sees the whole batch).
  Reference arm: the reference's own TP Transformer with its
  MLPTensorParallel resized to 5632 (it hard-codes the hidden size), without
  sequence parallel: its SP gather calls ``dist.all_gather_single``, which
  torch 2.11 does not provide.
* ``moe``: 12 layers, d_model 768, 12 heads x 64, 8 SwiGLU experts of
  hidden 1536 in every layer, softmax top-2 router with load-balancing loss and
  capacity factor 1.25, vocab 50304, seq_len 1024, global batch 64. Experts
  sharded over N ranks (EP=N), the rest data parallel (each rank 64/N
  sequences). Reference arm: its only router (sigmoid top-2 with bias balancing,
  no capacity limit, no auxiliary loss) and its only EP layout (one expert per
  rank, every rank processes the whole replicated batch), so N must be 8.
* ``cppp``: 16 layers split over PP=2 stages (GPipe, 8 microbatches), d_model
  1024, 16 heads x 64, SwiGLU 2816, vocab 50304, seq_len 16384, global batch 8,
  context parallel CP=N/2 inside each stage. The reference forbids pipeline +
  context parallel together, so its arm prints ``unavailable``.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402  (timing, clocks and process-group helpers)

VOCAB = 50304


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--config", choices=("tp", "moe", "cppp"), required=True)
    p.add_argument("--impl", choices=("abacus", "reference"), default="abacus")
    p.add_argument("--gpus", type=int, default=None)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--precision", choices=("fp32", "tf32"), default="fp32")
    p.add_argument("--global-batch", type=int, default=None)
    p.add_argument("--seq-len", type=int, default=None)
    p.add_argument("--layers", type=int, default=None, help="override the layer count (smoke runs only)")
    return p.parse_args()


DEFAULTS = {"tp": (16, 2048), "moe": (64, 1024), "cppp": (8, 16384)}


# ---------------------------------------------------------------------- abacus
def build_abacus(cfg, args, world, device):
    from abacus_b200.ops import precision
    from abacus_b200.parallel import mesh
    from abacus_b200.trainer import Trainer

    precision.set_precision(args.precision)
    torch.manual_seed(0)
    if cfg == "tp":
        from abacus_b200.transformer import Transformer

        if world > 1:
            mesh.init_mesh(tp=world)
        model = Transformer(dim=2048, n_heads=16, head_dim=128, n_blocks=args.layers or 24, vocab_size=VOCAB,
                            tensor_parallel=world > 1, sequence_parallel=world > 1, hidden_dim=5632)
        return Trainer(model, None, total_steps=1000, device=device), "tp%d+sp" % world, True
    if cfg == "moe":
        from abacus_b200.distributed.data_parallel import DataParallel
        from abacus_b200.transformer_moe import TransformerMoe

        if world > 1:
            mesh.init_mesh(dp=world, ep=world)
        model = TransformerMoe(768, 12, 64, args.layers or 12, VOCAB, 8, 2, hidden_dim=1536, router="softmax",
                               capacity_factor=1.25, expert_parallel=world > 1, expert_data_parallel=world > 1)
        parallel = None
        if world > 1:
            model = model.to(device)
            expert_params = [p for n, p in model.named_parameters() if ".moe.w_" in n]
            parallel = DataParallel(model, exclude=expert_params, token_weighted=False)
        return Trainer(model, parallel, total_steps=1000, device=device), "ep%d+dp%d" % (world, world), False
    # cppp
    from abacus_b200.parallel.pipeline_parallel import PipelineParallel
    from abacus_b200.transformer import PipelineStage

    if world % 2 != 0:
        raise SystemExit("cppp needs an even number of GPUs (PP=2 x CP=N/2)")
    cp = world // 2
    mesh.init_mesh(pp=2, cp=cp)
    pp_rank, _ = mesh.rank_and_world_size("pp")
    model = PipelineStage(1024, 16, 64, args.layers or 16, VOCAB, pp_rank, 2, hidden_dim=2816,
                          context_parallel=cp > 1)
    pipeline = PipelineParallel(model, n_microbatches=8)
    return Trainer(model, None, pipeline=pipeline, total_steps=1000, device=device), "pp2xcp%d" % cp, True


# ---------------------------------------------------------------------- reference
def build_reference(cfg, args, world, device):
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "abacus")):
        return None, "reference not installed in baseline/_ref", None, None
    if cfg == "cppp":
        return None, ("the reference forbids pipeline parallel with context parallel "
                      "(abacus/trainer.py raises), so PP=2 x CP cannot run"), None, None
    sys.path.insert(0, ref)
    from abacus.trainer import Trainer  # noqa: PLC0415

    torch.manual_seed(0)
    if cfg == "tp":
        from abacus.mlp import MLPTensorParallel  # noqa: PLC0415
        from abacus.transformer import Transformer  # noqa: PLC0415

        # The reference's sequence-parallel gather calls dist.all_gather_single,
        # which this torch does not have, so its arm runs TP without SP.
        model = Transformer(dim=2048, n_heads=16, head_dim=128, n_blocks=args.layers or 24, vocab_size=VOCAB,
                            tensor_parallel=world > 1, sequence_parallel=False)
        if world > 1:
            for block in model.blocks:
                block.mlp = MLPTensorParallel(2048, 5632, sequence_parallel=False)
        else:
            from abacus.mlp import MLP  # noqa: PLC0415

            for block in model.blocks:
                block.mlp = MLP(2048, 5632)
        return Trainer(model.to(device), total_steps=1000), None, "tp%d (no SP)" % world, True
    if world not in (1, 8):
        return None, "the reference's expert parallel keeps one expert per rank: 8 experts need 1 or 8 ranks", None, None
    from abacus.transformer_moe import TransformerMoe  # noqa: PLC0415

    model = TransformerMoe(768, 12, 64, args.layers or 12, VOCAB, 8, 2, hidden_dim=1536, expert_parallel=world > 1)
    return Trainer(model.to(device), total_steps=1000), None, "ep%d (replicated batch)" % world, True


def main():
    args = parse_args()
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    rank, world, local, device = bench.dist_setup(args.gpus or world_env)
    gb, sl = DEFAULTS[args.config]
    gb = args.global_batch or gb
    sl = args.seq_len or sl
    if args.impl == "reference":
        trainer, why, parallelism, replicated = build_reference(args.config, args, world, device)
        if trainer is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "config": args.config, "unavailable": why}), flush=True)
            if world > 1:
                dist.destroy_process_group()
            return
    else:
        trainer, parallelism, replicated = build_abacus(args.config, args, world, device)
    # replicated: every rank feeds the whole global batch (TP, pipeline + CP
    # stage inputs, reference EP); otherwise each rank gets global/N sequences.
    per_rank = gb if replicated else gb // world
    seed = 0 if replicated else 1_000_003 * rank
    gen = torch.Generator().manual_seed(seed)
    batches = [torch.randint(0, VOCAB, (per_rank, sl), generator=gen, dtype=torch.long).to(device) for _ in range(2)]

    def step(tokens):
        trainer.step(tokens)

    for i in range(args.warmup):
        step(batches[i % 2])
    torch.cuda.synchronize()
    sampler = bench.ClockSampler() if local == 0 else None
    if sampler:
        sampler.start()
    ms = bench.timed_steps(step, batches, args.steps, world, device)
    clocks = sampler.stop(list(range(world))) if sampler else None
    tokens = gb * sl * args.steps
    mem = torch.tensor([torch.cuda.max_memory_allocated(device) / 2**30], device=device)
    if world > 1:
        dist.all_reduce(mem, op=dist.ReduceOp.MAX)
    if rank == 0:
        line = {
            "metric": "train tokens/sec, whole box, device-timed max over ranks",
            "config": args.config,
            "value": tokens / (ms / 1000.0),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "global_batch": gb,
            "seq_len": sl,
            "layers": args.layers,
            "parallelism": parallelism,
            "dtype": args.precision if args.impl == "abacus" else "fp32",
            "max_mem_gib": round(float(mem), 1),
            "clocks": clocks,
            "data": "synthetic",
        }
        if args.impl == "reference":
            line["impl"] = "reference"
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
