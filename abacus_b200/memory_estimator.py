"""Analytic device-memory estimate for training a dense GPT
(``scripts/memory_estimator.py`` in the reference, which models fp32
parameters, gradients, Adam moments and activations including the O(L^2)
materialised scores).

Here the attention is flash-style (no score matrix; saved per layer: q, k, v,
output and log-sum-exp) and the cross entropy is fused (one logits chunk
instead of the full (T, V) logits), so activations are linear in L.

    python -m abacus_b200.memory_estimator --dim 768 --heads 12 --head-dim 64 --blocks 12 \\
        --hidden 2048 --vocab 50304 --batch 64 --seq-len 1024 [--dp 8 --zero 3]
"""
from __future__ import annotations

import argparse

GB = 1024**3


def estimate(dim, heads, head_dim, blocks, hidden, vocab, batch, seq_len, dp=1, zero=0, ce_chunk=8192):
    hk = heads * head_dim
    per_block = 3 * dim * hk + hk * dim + 3 * dim * hidden + 2 * dim + 2 * head_dim
    params = blocks * per_block + 2 * vocab * dim + dim
    b = 4  # fp32
    weights = params * b / (dp if zero >= 3 else 1)
    grads = params * b / (dp if zero >= 2 else 1)
    moments = 2 * params * b / (dp if zero >= 1 else 1)
    tokens = batch * seq_len
    # Saved per block: block input, 2 norm outputs, qkv, rotated q/k, attention
    # output + lse, post-attention residual, gate / up / silu(gate)*up.
    act_block = tokens * (dim * 4 + 3 * hk + 2 * hk + hk + heads + 3 * hidden) * b
    activations = blocks * act_block + tokens * dim * b * 2
    ce = min(ce_chunk, tokens) * vocab * b + vocab * dim * b + tokens * dim * b
    total = weights + grads + moments + activations + ce
    return {
        "params_M": params / 1e6,
        "weights_GB": weights / GB,
        "grads_GB": grads / GB,
        "adam_GB": moments / GB,
        "activations_GB": activations / GB,
        "cross_entropy_GB": ce / GB,
        "total_GB": total / GB,
    }


def main() -> None:
    p = argparse.ArgumentParser(description="Estimate training memory per GPU")
    for name, default in (("dim", 768), ("heads", 12), ("head-dim", 64), ("blocks", 12), ("hidden", 2048),
                          ("vocab", 50304), ("batch", 64), ("seq-len", 1024), ("dp", 1), ("zero", 0)):
        p.add_argument(f"--{name}", type=int, default=default)
    a = p.parse_args()
    est = estimate(a.dim, a.heads, a.head_dim, a.blocks, a.hidden, a.vocab, a.batch // a.dp, a.seq_len, a.dp, a.zero)
    for k, v in est.items():
        print(f"{k:>18}: {v:10.2f}")


if __name__ == "__main__":
    main()
