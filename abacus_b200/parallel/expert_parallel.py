"""Collectives for expert parallelism.

Semantics follow ``abacus/distributed/expert_parallel.py``:

* ``shard_counts`` (``:16-19``): contiguous token shards, remainder first.
* ``exchange_counts`` (``:22-26``): all-to-all of per-rank counts.
* ``_AllToAll`` (``:29-59``): variable-size exchange; backward swaps splits.
* ``_GatherTokenShards`` (``:62-86``): all-gather-v of the shard outputs;
  backward keeps this rank's slice.
* ``_SumReplicatedGrads`` (``:89-102``): identity forward, all-reduce backward.

The all-gather-v is a real ``all_gather_into_tensor`` of max-size padded
shards (the reference emulates it with an all-to-all of a P-times repeated
tensor). All collectives use the "ep" group of the installed mesh (the world
group without one).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from abacus_b200.parallel import mesh as _mesh

DIM = "ep"


def _rank_and_world_size(dim: str = DIM) -> tuple[int, int]:
    return _mesh.rank_and_world_size(dim)


def shard_counts(tokens: int, world_size: int) -> list[int]:
    """Contiguous token shards"""
    base, extra = divmod(tokens, world_size)
    return [base + (1 if rank < extra else 0) for rank in range(world_size)]


def exchange_counts(input_splits: torch.Tensor, dim: str = DIM) -> torch.Tensor:
    """One count per rank. output[i] is how many rows rank i sends here."""
    output_splits = torch.empty_like(input_splits)
    dist.all_to_all_single(output_splits, input_splits.contiguous(), group=_mesh.group_for(dim))
    return output_splits


class _AllToAll(torch.autograd.Function):
    """Variable-size token exchange. Backward swaps the split directions."""

    @staticmethod
    def forward(ctx, tokens, input_splits, output_splits, dim: str = DIM):
        ctx.input_splits = [int(s) for s in input_splits.tolist()]
        ctx.output_splits = [int(s) for s in output_splits.tolist()]
        ctx.dim = dim
        out = tokens.new_empty(sum(ctx.output_splits), *tokens.shape[1:])
        dist.all_to_all_single(
            out,
            tokens.detach().contiguous(),
            output_split_sizes=ctx.output_splits,
            input_split_sizes=ctx.input_splits,
            group=_mesh.group_for(dim),
        )
        return out

    @staticmethod
    def backward(ctx, grad):
        out = grad.new_empty(sum(ctx.input_splits), *grad.shape[1:])
        dist.all_to_all_single(
            out,
            grad.detach().contiguous(),
            output_split_sizes=ctx.input_splits,
            input_split_sizes=ctx.output_splits,
            group=_mesh.group_for(ctx.dim),
        )
        return out, None, None, None


class _GatherTokenShards(torch.autograd.Function):
    @staticmethod
    def forward(ctx, local_SD, counts, dim: str = DIM):
        rank, world = _rank_and_world_size(dim)
        ctx.rank = rank
        ctx.counts = [int(c) for c in counts.tolist()]
        ctx.offset = sum(ctx.counts[:rank])
        if world == 1:
            return local_SD
        width = max(ctx.counts)
        padded = local_SD.new_zeros((width, *local_SD.shape[1:]))
        padded[: local_SD.shape[0]] = local_SD.detach()
        gathered = padded.new_empty((world * width, *local_SD.shape[1:]))
        dist.all_gather_into_tensor(gathered, padded, group=_mesh.group_for(dim))
        gathered = gathered.view(world, width, *local_SD.shape[1:])
        return torch.cat([gathered[r, : ctx.counts[r]] for r in range(world)], dim=0)

    @staticmethod
    def backward(ctx, grad_TD):
        count = ctx.counts[ctx.rank]
        return grad_TD[ctx.offset : ctx.offset + count], None, None


class _SumReplicatedGrads(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tensor, dim: str = DIM):
        ctx.dim = dim
        return tensor

    @staticmethod
    def backward(ctx, grad):
        out = grad.detach().clone()
        _, world = _rank_and_world_size(ctx.dim)
        if world > 1:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=_mesh.group_for(ctx.dim))
        return out, None
