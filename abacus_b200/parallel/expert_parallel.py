"""Collectives for expert parallelism.

Semantics follow ``abacus/distributed/expert_parallel.py``:

* ``shard_counts`` (``:16-19``): contiguous token shards, remainder first
  (closed form here).
* ``exchange_counts`` (``:22-26``): receive counts from send counts (here the
  column of an all-gathered send-count matrix).
* ``_AllToAll`` (``:29-59``): variable-size exchange whose adjoint is the
  swapped exchange.
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
    """Split ``tokens`` rows into ``world_size`` contiguous runs; the first
    ``tokens % world_size`` runs are one row longer."""
    return [(tokens + world_size - 1 - r) // world_size for r in range(world_size)]


def exchange_counts(input_splits: torch.Tensor, dim: str = DIM) -> torch.Tensor:
    """Receive counts from send counts: entry i of the result is the number of
    rows rank i sends to this rank.

    Every rank contributes its send-count vector to a (P, P) matrix whose row
    r is rank r's sends; this rank's receive counts are the matrix's column.
    """
    rank, world = _rank_and_world_size(dim)
    sends = input_splits.reshape(-1).contiguous()
    if world == 1:
        return sends.clone()
    matrix = sends.new_empty(world * sends.numel())
    dist.all_gather_into_tensor(matrix, sends, group=_mesh.group_for(dim))
    return matrix.view(world, -1)[:, rank].contiguous()


def _as_sizes(counts) -> list[int]:
    return [int(c) for c in (counts.tolist() if torch.is_tensor(counts) else counts)]


def _exchange_rows(rows: torch.Tensor, send: list[int], recv: list[int], dim: str) -> torch.Tensor:
    out = rows.new_empty((sum(recv), *rows.shape[1:]))
    dist.all_to_all_single(out, rows.contiguous(), output_split_sizes=recv, input_split_sizes=send,
                           group=_mesh.group_for(dim))
    return out


class _AllToAll(torch.autograd.Function):
    """Row exchange with per-peer sizes (``send[i]`` rows go to rank i,
    ``recv[i]`` arrive from it). The exchange is linear and its adjoint is the
    same exchange with the size lists swapped, which is the backward."""

    @staticmethod
    def forward(ctx, tokens, input_splits, output_splits, dim: str = DIM):
        send, recv = _as_sizes(input_splits), _as_sizes(output_splits)
        ctx.adjoint = (recv, send, dim)
        return _exchange_rows(tokens.detach(), send, recv, dim)

    @staticmethod
    def backward(ctx, grad):
        send, recv, dim = ctx.adjoint
        return _exchange_rows(grad.detach(), send, recv, dim), None, None, None


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
