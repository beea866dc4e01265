"""Flagship training benchmark: ~125M dense GPT.

Model: 12 layers, d_model 768, 12 heads x 64, SwiGLU hidden 2048, RoPE,
QK-norm, vocab 50304, untied embeddings, fp32 parameters. Data: synthetic
uniform-random int64 tokens (seed 0), seq_len 1024, global batch 64
sequences (64 / N per rank; strong scaling). Data parallel for N > 1, one
process per GPU: by default the fused peer-memory gradient reduce + AdamW +
parameter broadcast kernels under backward (``--dp fused``); ``--dp nccl``
runs bucketed NCCL all-reduce + AdamW, ``--dp zero3`` ZeRO-3 with NVLink push
all-gathers and a fused reduce-scatter + AdamW, ``--dp zero3-nccl`` ZeRO-3 on
NCCL.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl abacus|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

``value``: training tokens/s of the whole job, device-timed with CUDA events
around exactly K steps (barrier + synchronize on both sides), max over ranks.
Inputs are resident on the device; every step's activations (several GB) are
far larger than the 126 MB L2, so no explicit flush is needed.
``e2e``: the same metric through the public API with the per-step host work
included: each step copies its batch from pinned host memory to the device
and reads the loss back to the host (``loss.item()``).

``--impl reference`` runs the unmodified reference framework (installed in
baseline/_ref) through its own public API on the same model/config, with the
MLP hidden size set to 2048 by assigning ``abacus.mlp.MLP(768, 2048)`` to each
block (the reference hard-codes 4*dim).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
BASELINE_TOKENS_PER_S = None  # the reference publishes no throughput numbers

MODEL = dict(dim=768, n_heads=12, head_dim=64, n_blocks=12, vocab_size=50304)
HIDDEN = 2048
SEQ_LEN = 1024
GLOBAL_BATCH = 64


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("abacus", "reference"), default="abacus")
    p.add_argument("--precision", choices=("fp32", "tf32"), default="fp32")
    p.add_argument("--global-batch", type=int, default=GLOBAL_BATCH)
    p.add_argument("--seq-len", type=int, default=SEQ_LEN)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--dp", choices=("fused", "nccl", "zero3", "zero3-nccl"), default="fused",
                   help="N>1: fused peer-memory reduce+AdamW kernel under backward, NCCL bucketed all-reduce + "
                        "AdamW, ZeRO-3 / FSDP with push all-gathers and a fused reduce-scatter + AdamW, or "
                        "ZeRO-3 on NCCL")
    return p.parse_args()


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while running."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self):
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL,
            )
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self, gpus: list[int]):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in gpus:
                    continue
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
            "reasons": sorted(reasons),
            "samples": len(rows),
        }


# ---------------------------------------------------------------------- setup
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    return rank, world, local, device


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed_steps(step_fn, batches, steps, world, device):
    """Device time (ms) of exactly `steps` calls, max over ranks."""
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        step_fn(batches[i % len(batches)])
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return max_over_ranks(start.elapsed_time(end), world, device)


# ---------------------------------------------------------------------- arms
def build_abacus(args, world, device):
    sys.path.insert(0, ROOT)
    from abacus_b200.ops import precision
    from abacus_b200.distributed.data_parallel import DataParallel, FusedDataParallel, FusedZero3
    from abacus_b200.trainer import Trainer
    from abacus_b200.transformer import Transformer

    precision.set_precision(args.precision)
    torch.manual_seed(0)
    model = Transformer(**MODEL, hidden_dim=HIDDEN)
    parallel = None
    if world > 1:
        model = model.to(device)
        if args.dp == "fused":
            parallel = FusedDataParallel(model)
        elif args.dp == "zero3":
            parallel = FusedZero3(model)
        else:
            parallel = DataParallel(model, stage=3 if args.dp == "zero3-nccl" else 0)
    trainer = Trainer(model, parallel, total_steps=args.warmup + 2 * args.steps + 2)
    return trainer


def build_reference(args, world, device):
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "abacus")):
        return None, "reference not installed in baseline/_ref"
    if world > 1 and args.dp in ("zero3", "zero3-nccl"):
        return None, ("the reference's ZeRO-3 calls dist.all_gather_single / reduce_scatter_single, "
                      "which torch 2.11 does not provide")
    sys.path.insert(0, ref)
    from abacus.distributed.data_parallel import DataParallel  # noqa: PLC0415
    from abacus.mlp import MLP  # noqa: PLC0415
    from abacus.trainer import Trainer  # noqa: PLC0415
    from abacus.transformer import Transformer  # noqa: PLC0415

    torch.manual_seed(0)
    model = Transformer(**MODEL)
    for block in model.blocks:
        block.mlp = MLP(MODEL["dim"], HIDDEN)
    parallel = DataParallel(model.to(device), stage=0) if world > 1 else None
    trainer = Trainer(model, parallel, total_steps=args.warmup + 2 * args.steps + 2)
    return trainer, None


def abacus_launches():
    try:
        from abacus_b200.ops._ext import ext

        return ext().launch_count()
    except Exception:  # noqa: BLE001
        return None


def main():
    args = parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    rank, world, local, device = dist_setup(args.gpus)
    if args.global_batch % world != 0:
        raise SystemExit("global batch must divide over the GPUs")
    per_rank = args.global_batch // world
    impl = args.impl
    if impl == "reference":
        trainer, why = build_reference(args, world, device)
        if trainer is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": why}))
            return
    else:
        trainer = build_abacus(args, world, device)

    gen = torch.Generator().manual_seed(0 + 1_000_003 * rank)
    host_batches = [
        torch.randint(0, MODEL["vocab_size"], (per_rank, args.seq_len), generator=gen, dtype=torch.long).pin_memory()
        for _ in range(2)
    ]
    dev_batches = [b.to(device) for b in host_batches]

    def step(tokens):
        trainer.step(tokens)

    # Warm-up (not timed).
    for i in range(args.warmup):
        step(dev_batches[i % 2])
    torch.cuda.synchronize()

    sampler = ClockSampler() if local == 0 else None
    if sampler:
        sampler.start()
    launches_before = abacus_launches() if impl == "abacus" else None
    ms = timed_steps(step, dev_batches, args.steps, world, device)
    launches = None
    if impl == "abacus" and launches_before is not None:
        launches = abacus_launches() - launches_before
    clocks = sampler.stop(list(range(world))) if sampler else None

    tokens_per_step = args.global_batch * args.seq_len
    value = tokens_per_step * args.steps / (ms / 1000.0)

    e2e = None
    if not args.no_e2e:
        def e2e_step(host_tokens):
            loss, _ = trainer.step(host_tokens)  # public API: pinned host batch in, H2D inside
            loss.item()  # D2H read of the step's result

        e2e_ms = timed_steps(e2e_step, host_batches, args.steps, world, device)
        e2e = {
            "value": tokens_per_step * args.steps / (e2e_ms / 1000.0),
            "unit": "tokens/s",
            "h2d_bytes_per_step": per_rank * args.seq_len * 8,
            "d2h_bytes_per_step": 4,
        }
    if rank == 0:
        line = {
            "metric": "train tokens/sec, whole box, device-timed max over ranks",
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None if BASELINE_TOKENS_PER_S is None else value / BASELINE_TOKENS_PER_S,
            "dtype": "fp32" if args.precision == "fp32" else "tf32",
            "data": "synthetic uniform-random int64 tokens (seed 0), random-init weights",
            "config": {
                "model": "dense GPT ~125M: 12L d768 12x64 heads, SwiGLU 2048, RoPE, QK-norm, vocab 50304",
                "global_batch": args.global_batch,
                "seq_len": args.seq_len,
                "parallelism": (f"zero3-dp{world}" if args.dp.startswith("zero3") else f"dp{world}")
                if world > 1 else "single",
                "dp_comm": None if world == 1 else (
                    "fused NVLink peer-memory gradient reduce + AdamW + broadcast per bucket under backward"
                    if impl == "abacus" and args.dp == "fused"
                    else ("NVLink push all-gather per unit + fused reduce-scatter / AdamW under backward (ZeRO-3)"
                          if impl == "abacus" and args.dp == "zero3"
                          else ("NCCL all-gather / reduce-scatter per unit (ZeRO-3)" if args.dp == "zero3-nccl"
                                else "NCCL all-reduce, then AdamW"))),
                "l2": "inputs/activations larger than L2 (no flush needed)",
                "compute": "3xTF32 split precision on tcgen05 (fp32 accuracy)" if args.precision == "fp32" and impl == "abacus"
                else ("tf32 tcgen05" if impl == "abacus" else "reference: torch fp32 (TF32 off)"),
            },
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if impl == "reference":
            line["impl"] = "reference"
        print(json.dumps(line), flush=True)
    if world > 1:
        parallel = getattr(trainer, "parallel", None)
        if hasattr(parallel, "check"):
            parallel.check()
        torch.cuda.synchronize()
        dist.barrier()
        if hasattr(parallel, "release"):
            parallel.release()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
