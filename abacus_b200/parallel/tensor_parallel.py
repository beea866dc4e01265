"""Autograd-aware collectives for Megatron tensor / sequence parallelism.

Semantics follow ``abacus/distributed/tensor_parallel.py``:

* ``_SumOutputs`` (g): all-reduce forward, identity backward (``:11-21``).
* ``_AllReduceGrads`` (f): identity forward, all-reduce backward (``:102-112``).
* ``_GatherFromSequenceParallel``: all-gather the sequence shard forward,
  reduce-scatter backward (``:55-64``).
* ``_ReduceScatterToSequenceParallel``: the mirror image (``:79-88``).
* ``_ScatterToSequenceParallel``: slice forward, all-gather backward (``:91-99``).
* ``_GatherReplicated``: all-gather forward, slice backward (``:67-76``).

Differences from the reference: every collective takes the "tp" group of the
installed mesh (the world group without one), and the sequence dimension is
gathered in place with ``all_gather_into_tensor`` on a (P, B, l, D) buffer
followed by one permute, instead of transposing to sequence-first both before
and after the collective.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from abacus_b200.parallel import mesh as _mesh

DIM = "tp"


def _rank_and_world_size(dim: str = DIM) -> tuple[int, int]:
    return _mesh.rank_and_world_size(dim)


def _group(dim: str = DIM):
    return _mesh.group_for(dim)


def all_gather_sequence(x_BlD: torch.Tensor, dim: str = DIM) -> torch.Tensor:
    """(B, L/P, ...) shard -> (B, L, ...) in rank order along the sequence."""
    _, world = _rank_and_world_size(dim)
    if world == 1:
        return x_BlD
    local = x_BlD.detach().contiguous()
    out = local.new_empty((world * local.shape[0], *local.shape[1:]))
    dist.all_gather_into_tensor(out, local, group=_group(dim))
    # (P*B, l, ...) -> (P, B, l, ...) -> (B, P, l, ...) -> (B, L, ...)
    out = out.view(world, *local.shape).movedim(0, 1)
    return out.reshape(local.shape[0], world * local.shape[1], *local.shape[2:])


def reduce_scatter_sequence(x_BLD: torch.Tensor, dim: str = DIM) -> torch.Tensor:
    """Sum partial (B, L, ...) over the group, keep this rank's (B, L/P, ...)."""
    _, world = _rank_and_world_size(dim)
    if world == 1:
        return x_BLD
    b, length = x_BLD.shape[0], x_BLD.shape[1]
    if length % world != 0:
        raise ValueError(f"sequence length {length} is not divisible by world size {world}")
    local_len = length // world
    chunks = x_BLD.detach().reshape(b, world, local_len, *x_BLD.shape[2:]).movedim(1, 0).contiguous()
    out = chunks.new_empty(chunks.shape[1:])
    dist.reduce_scatter_tensor(out, chunks.view(world * b, *chunks.shape[2:]), op=dist.ReduceOp.SUM, group=_group(dim))
    return out


def slice_sequence(x_BLD: torch.Tensor, dim: str = DIM) -> torch.Tensor:
    rank, world = _rank_and_world_size(dim)
    if world == 1:
        return x_BLD
    return x_BLD.detach().chunk(world, dim=1)[rank].contiguous()


def all_reduce_sum(x: torch.Tensor, dim: str = DIM) -> torch.Tensor:
    out = x.detach().clone()
    _, world = _rank_and_world_size(dim)
    if world > 1:
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=_group(dim))
    return out


class _SumOutputs(torch.autograd.Function):
    @staticmethod
    def forward(ctx, partial_BLD: torch.Tensor, dim: str = DIM) -> torch.Tensor:
        return all_reduce_sum(partial_BLD, dim)

    @staticmethod
    def backward(ctx, grad_BLD: torch.Tensor):
        return grad_BLD, None


class _GatherFromSequenceParallel(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_BlD: torch.Tensor, dim: str = DIM) -> torch.Tensor:
        ctx.dim = dim
        return all_gather_sequence(x_BlD, dim)

    @staticmethod
    def backward(ctx, grad_BLD: torch.Tensor):
        return reduce_scatter_sequence(grad_BLD, ctx.dim), None


class _GatherReplicated(torch.autograd.Function):
    """All-gather after the final norm; the replicated logits' gradient is
    sliced back, not summed."""

    @staticmethod
    def forward(ctx, x_BlD: torch.Tensor, dim: str = DIM) -> torch.Tensor:
        ctx.dim = dim
        return all_gather_sequence(x_BlD, dim)

    @staticmethod
    def backward(ctx, grad_BLD: torch.Tensor):
        return slice_sequence(grad_BLD, ctx.dim), None


class _ReduceScatterToSequenceParallel(torch.autograd.Function):
    @staticmethod
    def forward(ctx, partial_BLD: torch.Tensor, dim: str = DIM) -> torch.Tensor:
        ctx.dim = dim
        return reduce_scatter_sequence(partial_BLD, dim)

    @staticmethod
    def backward(ctx, grad_BlD: torch.Tensor):
        return all_gather_sequence(grad_BlD.contiguous(), ctx.dim), None


class _ScatterToSequenceParallel(torch.autograd.Function):
    """Keep this rank's slice before the first block."""

    @staticmethod
    def forward(ctx, x_BLD: torch.Tensor, dim: str = DIM) -> torch.Tensor:
        ctx.dim = dim
        return slice_sequence(x_BLD, dim)

    @staticmethod
    def backward(ctx, grad_BlD: torch.Tensor):
        return all_gather_sequence(grad_BlD.contiguous(), ctx.dim), None


class _AllReduceGrads(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weight: torch.Tensor, dim: str = DIM) -> torch.Tensor:
        ctx.dim = dim
        return weight

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        return all_reduce_sum(grad, ctx.dim), None
