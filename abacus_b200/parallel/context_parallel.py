"""Llama-3 style all-gather-KV context parallelism with zigzag load balancing.

Semantics follow ``abacus/distributed/context_parallel.py``:

* ``zigzag_positions`` (``:7-18``): rank i keeps chunks i and 2P-1-i.
* ``_AllGatherSequenceBlock`` (``:33-53``): all-gather K or V along the
  sequence (dim 2 of (B, H, l, K)); backward reduce-scatters onto the owner.
* ``sum_parameter_gradients`` (``:56-66``): one flat all-reduce SUM of every
  parameter gradient (the CP loss is already divided by the global count).

The key positions of the gathered sequence are a closed-form function of the
zigzag layout, so ``all_gather_positions`` needs no collective: it is
computed locally (the reference all-gathers them, ``:21-30``).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from abacus_b200.parallel import mesh as _mesh

DIM = "cp"


def _rank_and_world_size(dim: str = DIM) -> tuple[int, int]:
    return _mesh.rank_and_world_size(dim)


def zigzag_positions(length: int, rank: int, world_size: int) -> torch.Tensor:
    """Rank i keeps chunk i and chunk 2*world_size-1-i, so causal work is balanced."""
    chunks = 2 * world_size
    if length % chunks != 0:
        raise ValueError(f"sequence length {length} is not divisible by {chunks}")
    chunk = length // chunks
    first = rank * chunk
    second = (chunks - 1 - rank) * chunk
    return torch.cat((torch.arange(first, first + chunk), torch.arange(second, second + chunk)))


def gathered_positions(local_length: int, world_size: int) -> torch.Tensor:
    """Global positions of the keys after an all-gather of every rank's zigzag shard."""
    total = local_length * world_size
    return torch.cat([zigzag_positions(total, r, world_size) for r in range(world_size)])


def all_gather_positions(positions: torch.Tensor, dim: str = DIM) -> torch.Tensor:
    _, world = _rank_and_world_size(dim)
    if world == 1:
        return positions
    return gathered_positions(positions.shape[0], world).to(positions.device)


class _AllGatherSequenceBlock(torch.autograd.Function):
    """All-gather K or V along the sequence. Backward sums grads onto the owner."""

    @staticmethod
    def forward(ctx, block_BHPK: torch.Tensor, dim: str = DIM) -> torch.Tensor:
        _, world = _rank_and_world_size(dim)
        ctx.world_size = world
        ctx.dim = dim
        if world == 1:
            return block_BHPK.detach().clone()
        local = block_BHPK.detach().contiguous()
        out = local.new_empty((world * local.shape[0], *local.shape[1:]))
        dist.all_gather_into_tensor(out, local, group=_mesh.group_for(dim))
        b, h, l, k = local.shape
        return out.view(world, b, h, l, k).permute(1, 2, 0, 3, 4).reshape(b, h, world * l, k)

    @staticmethod
    def backward(ctx, grad_BHPK: torch.Tensor):
        if ctx.world_size == 1:
            return grad_BHPK, None
        world = ctx.world_size
        b, h, length, k = grad_BHPK.shape
        chunks = grad_BHPK.reshape(b, h, world, length // world, k).permute(2, 0, 1, 3, 4).contiguous()
        out = chunks.new_empty(chunks.shape[1:])
        dist.reduce_scatter_tensor(out, chunks.view(world * b, h, length // world, k), op=dist.ReduceOp.SUM,
                                   group=_mesh.group_for(ctx.dim))
        return out, None


def sum_parameter_gradients(model: torch.nn.Module, dim: str = DIM) -> None:
    grads = [param.grad for param in model.parameters() if param.grad is not None]
    if not grads:
        raise RuntimeError("backward produced no gradients")
    _, world = _rank_and_world_size(dim)
    if world == 1:
        return
    flat = torch.cat([grad.reshape(-1) for grad in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=_mesh.group_for(dim))
    offset = 0
    for grad in grads:
        numel = grad.numel()
        grad.copy_(flat[offset : offset + numel].view_as(grad))
        offset += numel
