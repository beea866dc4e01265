"""Shared command-line plumbing for the example trainers.

Flags common to every example follow the reference's (``--data``,
``--limit``, ``--liger``; ``examples/train_gpt_dp.py:87-96``) plus:

* ``--synthetic N``: N uniform-random documents instead of the tokenised
  pile-10k file (the benchmark data; no download needed);
* ``--precision {fp32,tf32}``: tensor-core precision of the CUDA kernels;
* ``--steps``: stop after this many steps.
"""
from __future__ import annotations

import argparse
import time
from pathlib import Path

import torch

from abacus_b200.kernels.liger import set_use_liger
from abacus_b200.ops import precision
from abacus_b200.utils.data import load_documents, padded_batches, select_documents
from abacus_b200.utils.dist import dist_env_vars, init_process_group, rank, shutdown, world_size

DEFAULT_DATA = Path(__file__).resolve().parents[2] / "data" / "pile-10k.pt"


def base_parser(description: str) -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=description)
    p.add_argument("--data", type=Path, default=DEFAULT_DATA)
    p.add_argument("--limit", type=int, default=None)
    p.add_argument("--liger", action="store_true", help="accepted for compatibility; CE always runs fused")
    p.add_argument("--synthetic", type=int, default=None, metavar="N", help="use N synthetic documents")
    p.add_argument("--synthetic-length", type=int, default=128)
    p.add_argument("--vocab-size", type=int, default=50304, help="vocabulary of synthetic data")
    p.add_argument("--precision", choices=("fp32", "tf32"), default="fp32")
    p.add_argument("--steps", type=int, default=None)
    p.add_argument("--phase-times", action="store_true",
                   help="print device time per step phase (forward / backward / sync / optimizer) and tokens/s")
    return p


def setup(args):
    """Process group (when launched by torchrun), device, precision flags."""
    from abacus_b200.trainer import get_device

    if args.limit is not None and args.limit < 1:
        raise ValueError(f"--limit must be at least 1, got {args.limit}")
    set_use_liger(args.liger)
    precision.set_precision(args.precision)
    device = get_device()
    distributed = dist_env_vars()
    if distributed:
        init_process_group("nccl" if device.type == "cuda" else "gloo", device)
    return device, distributed


def documents(args, rank_: int = 0, world: int = 1):
    """(documents, vocab_size) from --data or --synthetic."""
    if args.synthetic is not None:
        g = torch.Generator().manual_seed(0)
        docs = []
        for _ in range(args.synthetic):
            n = int(torch.randint(2, args.synthetic_length + 1, (1,), generator=g))
            docs.append(torch.randint(0, args.vocab_size, (n,), generator=g))
        return select_documents(docs, args.limit, rank_, world), args.vocab_size
    docs, vocab = load_documents(args.data)
    return select_documents(docs, args.limit, rank_, world), vocab


def run_loop(trainer, batches, total_steps, device, distributed, log_every: int = 1, on_step=None, max_steps=None):
    started = time.perf_counter()
    is_main = not distributed or rank() == 0
    for step, tokens in enumerate(batches, start=1):
        if max_steps is not None and step > max_steps:
            break
        loss, local = trainer.step(tokens.to(device))
        if on_step is not None:
            on_step(step, loss, local, tokens)
        elif is_main and step % log_every == 0:
            print(f"step {step}/{total_steps} loss {loss.item():.4f} batch {tokens.shape[0]} length {tokens.shape[1]}",
                  flush=True)
        tracer = getattr(trainer, "tracer", None)
        if tracer is not None and tracer.timing:
            times = tracer.times_ms()
            if is_main and step % log_every == 0:
                total = sum(times.values())
                rate = tokens.numel() / (total / 1e3) if total > 0 else 0.0
                parts = " ".join(f"{k} {v:.1f} ms" for k, v in times.items())
                print(f"  phases: {parts} | {rate:,.0f} tokens/s on this rank", flush=True)
    if is_main:
        print(f"Execution time {time.perf_counter() - started:.1f}", flush=True)


__all__ = ["base_parser", "setup", "documents", "padded_batches", "run_loop", "shutdown", "rank", "world_size"]
