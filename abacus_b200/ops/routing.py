"""Capacity-slot assignment of MoE routing (device side on CUDA)."""
from __future__ import annotations

import torch

from abacus_b200.ops._ext import ext


def expert_rank(flat_e: torch.Tensor, n_experts: int) -> torch.Tensor:
    """Rank of each assignment among the assignments to the same expert, in
    list order (its slot in the expert's capacity slab): one scan kernel on
    CUDA (``expert_rank_kernel``), a one-hot prefix sum on CPU."""
    if flat_e.is_cuda:
        flat = flat_e.to(torch.int64).contiguous()
        rank = torch.empty_like(flat)
        ext().expert_rank(flat, n_experts, rank)
        return rank
    onehot = torch.nn.functional.one_hot(flat_e, n_experts)
    return (onehot.cumsum(dim=0) * onehot).sum(dim=-1) - 1
