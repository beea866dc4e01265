"""Context parallel attention (Llama-3 style all-gather of K / V) with the
gather fused into the flash-attention kernel's K/V loads and the backward
reduce-scatter of dK / dV fused into the backward kernel's stores.

Reference semantics: ``abacus/distributed/context_parallel.py`` (each rank
holds a zigzag pair of sequence chunks; K and V of every rank are gathered,
queries attend by global position; dK / dV are summed back to the owners).
There the gather is an NCCL all-gather before attention and a reduce-scatter
after its backward. Here:

* forward: this rank's [K | V] rows are pushed into every CP rank's gathered
  buffer (``tp_push_rows``) and the flash kernel's CTAs start as soon as every
  owner published its epoch (``flash_attn_fwd_cp``), reading K / V tiles from
  the local gathered buffer with TMA;
* backward: the dK / dV tile of every 128 gathered keys is stored straight
  into its owner's staging slot over NVLink and counted
  (``flash_attn_bwd_cp``); the owner sums the slots in rank order
  (``tp_reduce_rows``).

Buffers are keyed per attention module and per call within a step, so the
microbatches of a pipeline step never share one; a bounded device barrier
over the CP group starts every step (``tp_fused.Workspace.begin_step``).
"""
from __future__ import annotations

import math
import os

import torch

from abacus_b200.ops import precision
from abacus_b200.ops._ext import ext
from abacus_b200.parallel import mesh, tp_fused

DIM = "cp"


def enabled() -> bool:
    return os.environ.get("ABACUS_CP_FUSED", "1") != "0"


def usable(x: torch.Tensor, local_len: int, head_dim: int) -> bool:
    _, world = mesh.rank_and_world_size(DIM)
    supported = head_dim in (32, 64) or (head_dim == 128 and precision.passes() == 1)
    return (enabled() and x.is_cuda and x.dtype == torch.float32 and 2 <= world <= 8 and local_len % 128 == 0
            and supported)


def begin_step(device: torch.device) -> None:
    tp_fused.begin_step(device, DIM)


class _CPAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, q_pos, k_pos, batch, heads, head_dim, key):
        ws = tp_fused.workspace(q.device, DIM)
        call = ws.call_key(key)
        hk = heads * head_dim
        local = k.shape[0] // batch
        world, rank = ws.world, ws.rank
        seq = local * world
        lq = q.shape[0] // batch
        kv = torch.cat((k, v), dim=1)
        gathered, spec = ws.push_gather(call + ".KV", kv, local, seq)
        flags, epoch, _, _, _ = spec
        out = torch.empty(q.shape[0], hk, device=q.device, dtype=torch.float32)
        lse = torch.empty(batch, heads, lq, device=q.device, dtype=torch.float32)
        scale = 1.0 / math.sqrt(head_dim)
        ext().flash_attn_fwd_cp(q, gathered[:, :hk], gathered[:, hk:], out, lse, batch, heads, head_dim, lq, seq,
                                scale, q_pos, k_pos, precision.passes(), [flags, epoch, world, rank])
        ctx.save_for_backward(q, gathered, out, lse, q_pos, k_pos)
        ctx.meta = (call, batch, heads, head_dim, lq, local, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, gathered, out, lse, q_pos, k_pos = ctx.saved_tensors
        call, batch, heads, head_dim, lq, local, scale = ctx.meta
        ws = tp_fused.workspace(q.device, DIM)
        ws._backward_seen = True
        world, rank = ws.world, ws.rank
        hk = heads * head_dim
        slot = batch * local * hk
        buf_k, ptrs_k = ws.buffer(call + ".dK", world * slot)
        buf_v, ptrs_v = ws.buffer(call + ".dV", world * slot)
        off = ws.slots(call + ".dKV")
        stage_k = buf_k[: world * slot].view(world, batch * local, hk)
        stage_v = buf_v[: world * slot].view(world, batch * local, hk)
        scatter = [local]
        scatter += [p + 4 * rank * slot for p in ptrs_k]
        scatter += [p + 4 * rank * slot for p in ptrs_v]
        scatter += [p + 4 * (off + rank) for p in ws.signal_ptrs]
        dq = torch.empty_like(q)
        ext().flash_attn_bwd_cp(q, gathered[:, :hk], gathered[:, hk:], out, dout.contiguous(), lse, dq,
                                stage_k[rank], stage_v[rank], batch, heads, head_dim, lq, local * world, scale,
                                q_pos, k_pos, precision.passes(), scatter)
        # Tiles each owner receives from this rank: its keys / 128, per head and sequence.
        target = ws.add_target(call + ".dKV", (local // 128) * heads * batch)
        counters = ws.signal[off : off + world]
        dk = torch.empty(batch * local, hk, device=q.device, dtype=torch.float32)
        dv = torch.empty_like(dk)
        ext().tp_reduce_rows(stage_k, world, counters, target, None, dk)
        ext().tp_reduce_rows(stage_v, world, counters, target, None, dv)
        return dq, dk, dv, None, None, None, None, None, None


def attention(q, k, v, batch, heads, head_dim, q_pos, k_pos, key):
    """Causal attention of this rank's queries (global positions ``q_pos``)
    over every CP rank's keys (``k_pos``, gathered rank order); q, k, v are
    this rank's (B*l, H*K) rows."""
    return _CPAttention.apply(q.contiguous(), k, v, q_pos, k_pos, batch, heads, head_dim, key)
