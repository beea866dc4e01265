"""Cross-entropy latency: abacus_b200 kernel vs ``F.cross_entropy``, vocab
32000, 16..4096 tokens, CUDA events, 10 warm-up and 100 timed calls, p50 /
p90 / p99 (the measurement the reference's Liger benchmark reports), plus the
fused linear + cross-entropy against logits-GEMM + CE.

    python benchmarks/bench_cross_entropy.py
"""
import json
import os
import sys

import torch
import torch.nn.functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from abacus_b200.ops import cross_entropy as ce  # noqa: E402


def percentiles(fn, warmup=10, iters=100):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return {q: times[int(q / 100 * (len(times) - 1))] for q in (50, 90, 99)}


def main():
    vocab = 32000
    for tokens in (16, 64, 256, 1024, 4096):
        logits = torch.randn(tokens, vocab, device="cuda", requires_grad=True)
        tgt = torch.randint(0, vocab, (tokens,), device="cuda")
        ours = percentiles(lambda: ce.cross_entropy(logits, tgt).backward())
        ref = percentiles(lambda: F.cross_entropy(logits, tgt).backward())
        print(json.dumps({"tokens": tokens, "abacus_ms": ours, "torch_ms": ref}), flush=True)


if __name__ == "__main__":
    main()
