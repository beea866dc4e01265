"""Device-timed GEMM benchmark: abacus_b200 tcgen05 kernels vs cuBLAS.

Shapes are the per-step GEMMs of the ~125M dense config (T = 65536 tokens,
d_model 768, SwiGLU hidden 2048, vocab 50304). Each case runs 3 warm-up and
`--iters` timed launches with CUDA events on the launching stream; an L2 flush
(a 256 MB write) separates timed launches.

    python benchmarks/bench_gemm.py [--iters 10] [--tokens 65536]
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from abacus_b200.ops import gemm, precision


def timed(fn, iters, flush):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.zero_()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    times.sort()
    return times[len(times) // 2]


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--iters", type=int, default=10)
    parser.add_argument("--tokens", type=int, default=65536)
    args = parser.parse_args()
    t = args.tokens
    flush = torch.empty(64 * 1024 * 1024, device="cuda")
    cases = [
        ("qkv x@W", (t, 768), (768, 2304), False, False),
        ("o-proj x@W", (t, 768), (768, 768), False, False),
        ("up x@W", (t, 768), (768, 2048), False, False),
        ("down x@W", (t, 2048), (2048, 768), False, False),
        ("dgrad dy@W^T", (t, 2048), (768, 2048), False, True),
        ("wgrad x^T@dy", (t, 768), (t, 2048), True, False),
        ("logits x@W", (8192, 768), (768, 50304), False, False),
    ]
    rows = []
    for name, sa, sb, ta, tb in cases:
        a = torch.randn(*sa, device="cuda")
        b = torch.randn(*sb, device="cuda")
        m = sa[1] if ta else sa[0]
        k = sa[0] if ta else sa[1]
        n = sb[0] if tb else sb[1]
        flops = 2.0 * m * n * k
        lhs = a.t() if ta else a
        rhs = b.t() if tb else b
        out = {}
        for mode in ("tf32", "fp32"):
            precision.set_precision(mode)
            ms = timed(lambda: gemm.matmul(a, b, trans_a=ta, trans_b=tb), args.iters, flush)
            out[f"abacus_{mode}_tflops"] = flops / ms / 1e9
        precision.set_precision("fp32")
        torch.backends.cuda.matmul.allow_tf32 = False
        ms = timed(lambda: lhs @ rhs, args.iters, flush)
        out["cublas_fp32_tflops"] = flops / ms / 1e9
        torch.backends.cuda.matmul.allow_tf32 = True
        ms = timed(lambda: lhs @ rhs, args.iters, flush)
        out["cublas_tf32_tflops"] = flops / ms / 1e9
        torch.backends.cuda.matmul.allow_tf32 = False
        rows.append({"case": name, "m": m, "n": n, "k": k, **{k2: round(v, 1) for k2, v in out.items()}})
        print(json.dumps(rows[-1]), flush=True)


if __name__ == "__main__":
    main()
