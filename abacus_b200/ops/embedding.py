"""Embedding lookup ``w[tokens]`` (``abacus/embedding.py:19-23``).

CUDA backward is deterministic: tokens are stably sorted and each run of equal
ids is summed in token order by one warp (no float atomics).
"""
from __future__ import annotations

import torch

from abacus_b200.ops._ext import ext


class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, weight):
        flat = tokens.reshape(-1).contiguous()
        out = torch.empty(flat.numel(), weight.shape[1], device=weight.device, dtype=weight.dtype)
        ext().embedding_fwd(flat, weight, out)
        ctx.save_for_backward(flat)
        ctx.vocab = weight.shape[0]
        ctx.shape = tokens.shape
        return out.view(*tokens.shape, weight.shape[1])

    @staticmethod
    def backward(ctx, grad):
        (flat,) = ctx.saved_tensors
        g = grad.reshape(flat.numel(), -1).contiguous()
        sorted_tok, perm = torch.sort(flat, stable=True)
        dw = torch.zeros(ctx.vocab, g.shape[1], device=g.device, dtype=g.dtype)
        ext().embedding_bwd(sorted_tok, perm, g, dw)
        return None, dw


def embedding(tokens: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    if not weight.is_cuda:
        return weight[tokens]
    return _Embedding.apply(tokens.to(weight.device), weight)
