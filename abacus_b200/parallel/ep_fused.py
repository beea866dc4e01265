"""Expert parallelism with the dispatch / combine all-to-all fused into the
router permutation and the expert GEMMs, over NVLink peer memory.

Reference semantics: ``abacus/distributed/expert_parallel.py:29-59`` and
``abacus/moe/moe.py`` (every (token, slot) assignment goes to the rank that
owns its expert, the expert's SwiGLU runs on its rows, the results come back
and each token sums its slots weighted by the router). The reference sorts
the rows by expert, exchanges them with an NCCL all-to-all (and a second one
back), then un-permutes. Here, per MoE layer:

* counts: one small all-gather of the per-expert assignment counts fixes every
  row's destination (slab of its expert on the owning rank, then source rank,
  then (token, slot) order) -- the only host sync, as in the reference;
* dispatch: ``ep_push_rows`` writes each assignment's row straight into its
  expert's slab on the owning rank (the permutation and the all-to-all are one
  pass) and records where its result must return;
* experts: the SwiGLU GEMM of each local expert starts once every rank's rows
  arrived (bounded wait in the GEMM), and the down-projection GEMM's epilogue
  stores every output row straight back into its source rank's return buffer;
* combine: ``ep_combine`` waits for all rows and sums each token's slots
  weighted by the router.

Backward mirrors it: the weighted output gradient is pushed to the experts'
slabs, the SwiGLU backward GEMM waits for it, and the dX GEMM's epilogue
returns each row to its source, which sums the slots. Router-weight gradients
are <dY_t, y_slot> from the returned rows.

With a capacity factor (``dispatch_combine_capacity``) the slabs are static
and nothing leaves the device: each expert's slab on its owner holds
``world * C`` rows, source rank r owning rows [r*C, (r+1)*C), where C is the
per-rank capacity of the router (the first C assignments of each expert in
(token, slot) order are kept, the rest dropped, exactly the router's capacity
rule). A row's destination is then a function of its own rank's routing only,
so there is no counts exchange and no host sync; the expert GEMMs have fixed
shapes. Unfilled slab rows carry a negative meta (their outputs are not
returned) and zero gradients; dropped assignments are credited to the return
counter by their source and get weight 0 in the combine.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from abacus_b200.ops import precision
from abacus_b200.ops._ext import ext
from abacus_b200.ops.routing import expert_rank
from abacus_b200.parallel import mesh, tp_fused

DIM = "ep"
_SINGLE, _SEG_K = 0, 2


def enabled() -> bool:
    return os.environ.get("ABACUS_EP_FUSED", "1") != "0"


def usable(x: torch.Tensor, hidden: int) -> bool:
    _, world = mesh.rank_and_world_size(DIM)
    return (enabled() and x.is_cuda and x.dtype == torch.float32 and 2 <= world <= 8 and x.shape[-1] % 4 == 0
            and hidden % 32 == 0)


def _plan(flat_e: torch.Tensor, n_experts: int, local_experts: int, ws):
    """Counts exchange and row placement. Returns host tables and device
    (dest_rank, dest_row) per assignment."""
    world, me = ws.world, ws.rank
    counts = torch.bincount(flat_e, minlength=n_experts)
    gathered = torch.empty(world * n_experts, dtype=counts.dtype, device=counts.device)
    dist.all_gather_into_tensor(gathered, counts, group=ws.group)
    c = gathered.view(world, n_experts).cpu()  # the one host sync per layer
    slab = c.sum(dim=0).view(world, local_experts)  # rows of (rank, local expert)
    base = torch.cumsum(slab, dim=1) - slab  # slab start inside its rank's buffer
    src_off = torch.cumsum(c, dim=0) - c  # rows of earlier source ranks in each expert slab
    table = base.reshape(-1) + src_off[me]  # start of my rows in each expert's slab
    order = torch.argsort(flat_e, stable=True)
    starts = torch.cumsum(counts, 0) - counts
    pos = torch.arange(flat_e.numel(), device=flat_e.device) - starts[flat_e[order]]
    within = torch.empty_like(pos)
    within[order] = pos
    dest_row = (table.to(flat_e.device)[flat_e] + within).to(torch.int32)
    dest_rank = torch.div(flat_e, local_experts, rounding_mode="floor").to(torch.int32)
    recv_rows = slab.sum(dim=1)
    sent_rows = c.sum(dim=1)
    return {
        "slab": slab[me].tolist(),
        "base": base[me].tolist(),
        "recv_max": int(recv_rows.max()),
        "sent_max": int(sent_rows.max()),
        "typical": int(sent_rows.max()),  # balanced routing: a rank receives what it sends
        "worst": int(sent_rows.sum()),  # every assignment routed to one rank
        "dest_rank": dest_rank.contiguous(),
        "dest_row": dest_row.contiguous(),
    }


def _capacity(needed: int, typical: int, worst: int) -> int:
    """Rows to allocate for a receive buffer. Every size change is a collective
    re-allocation, so grow with headroom: twice the balanced load at first,
    then twice what a step needed, never more than the worst case."""
    return min(worst, max(needed, 2 * typical, 2 * needed if needed > 2 * typical else 0))


def _push(ws, key, src, top_k, plan, scale):
    """Dispatch rows into every rank's buffer `key`; returns (rows, meta, wait spec)."""
    dim = src.shape[1]
    rows_cap = _capacity(plan["recv_max"], plan["typical"], plan["worst"])
    rows_buf, rows_ptrs = ws.buffer(key, max(1, rows_cap) * dim)
    meta_buf, meta_ptrs = ws.buffer(key + ".meta", max(1, rows_cap))
    off = ws.slots(key)
    epoch = ws.next_epoch(key)
    done = ws._done.get(key)
    if done is None:
        done = ws._done[key] = torch.zeros(1, dtype=torch.int32, device=src.device)
    flags = [p + 4 * (off + ws.rank) for p in ws.signal_ptrs]
    ext().ep_push_rows(src, top_k, plan["dest_rank"], plan["dest_row"], scale, rows_ptrs, meta_ptrs, flags, ws.rank,
                       epoch, done)
    wait = [ws.signal_ptrs[ws.rank] + 4 * off, 2, epoch, 1, ws.world, ws.rank]
    rows = rows_buf[: plan["recv_max"] * dim].view(plan["recv_max"], dim)
    meta = meta_buf[: max(1, plan["recv_max"])].view(torch.int32)
    return rows, meta, wait


def _return_target(ws, key, sent_max, dim):
    """Return buffer `key` on every rank (rows come back here) and its counter."""
    buf, ptrs = ws.buffer(key, max(1, sent_max) * dim)
    off = ws.slots(key)
    counters = [p + 4 * off for p in ws.signal_ptrs]
    return buf, ptrs, counters, ws.signal[off : off + 1]


class _EPFused(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weights, indices, w_gate, w_up, w_down, n_experts, key):
        ws = tp_fused.workspace(x.device, DIM)
        ws.begin_step()
        call = ws.call_key(key)
        n, dim = x.shape
        top_k = indices.shape[1]
        local_experts = w_gate.shape[0]
        hidden = w_gate.shape[2]
        passes = precision.passes()
        plan = _plan(indices.reshape(-1), n_experts, local_experts, ws)
        rows, meta, wait = _push(ws, call + ".X", x.contiguous(), top_k, plan, None)
        ret, ret_ptrs, counter_ptrs, counter = _return_target(ws, call + ".R", plan["sent_max"], dim)
        n_tiles = ext().gemm_n_tiles(dim, passes)
        saved = []
        for le in range(local_experts):
            m, start = plan["slab"][le], plan["base"][le]
            if m == 0:
                saved.append(None)
                continue
            xs = rows[start : start + m]
            g = torch.empty(m, hidden, device=x.device, dtype=torch.float32)
            u = torch.empty_like(g)
            h = torch.empty_like(g)
            ext().gemm_swiglu_tp(xs, w_gate[le], w_up[le], g, u, h, passes, wait)
            mrow = meta[start : start + m]
            scatter = [-1, mrow.data_ptr()] + list(ret_ptrs) + list(counter_ptrs)
            ext().gemm_out_tp(ret[: dim].view(1, dim), h, [w_down[le]], False, False, _SINGLE, 1.0, passes, None,
                              scatter)
            saved.append((g, u, h))
        target = ws.add_target(call + ".R", n * top_k * n_tiles)
        out = torch.empty(n, dim, device=x.device, dtype=torch.float32)
        ret_rows = ret[: n * top_k * dim].view(n * top_k, dim)
        ext().ep_combine(ret_rows, weights.contiguous(), top_k, counter, target, out)
        ctx.save_for_backward(weights, w_gate, w_up, w_down)
        ctx.saved = saved
        ctx.meta = (call, plan, n, dim, top_k, hidden, n_tiles)
        ctx.buffers = (rows, meta, ret_rows)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        weights, w_gate, w_up, w_down = ctx.saved_tensors
        call, plan, n, dim, top_k, hidden, n_tiles = ctx.meta
        rows, meta, ret_rows = ctx.buffers
        ws = tp_fused.workspace(grad_out.device, DIM)
        ws._backward_seen = True
        passes = precision.passes()
        grad_out = grad_out.contiguous()
        scale = weights.reshape(-1).contiguous()
        dy_rows, _, wait = _push(ws, call + ".dY", grad_out, top_k, plan, scale)
        dret, dret_ptrs, counter_ptrs, counter = _return_target(ws, call + ".dR", plan["sent_max"], dim)
        d_gate = torch.zeros_like(w_gate)
        d_up = torch.zeros_like(w_up)
        d_down = torch.zeros_like(w_down)
        for le, item in enumerate(ctx.saved):
            if item is None:
                continue
            g, u, h = item
            m, start = plan["slab"][le], plan["base"][le]
            dys = dy_rows[start : start + m]
            dgu = torch.empty(m, 2 * hidden, device=grad_out.device, dtype=torch.float32)
            ext().gemm_swiglu_bwd_tp(dys, w_down[le], g, u, dgu, passes, wait)
            scatter = [-1, meta[start : start + m].data_ptr()] + list(dret_ptrs) + list(counter_ptrs)
            ext().gemm_out_tp(dret[: dim].view(1, dim), dgu, [w_gate[le], w_up[le]], False, True, _SEG_K, 1.0,
                              passes, None, scatter)
            xs = rows[start : start + m]
            ext().gemm_out(d_gate[le], xs, [dgu[:, :hidden]], True, False, _SINGLE, 1.0, None, False, passes)
            ext().gemm_out(d_up[le], xs, [dgu[:, hidden:]], True, False, _SINGLE, 1.0, None, False, passes)
            ext().gemm_out(d_down[le], h, [dys], True, False, _SINGLE, 1.0, None, False, passes)
        dx_tiles = ext().gemm_n_tiles(dim, passes)
        target = ws.add_target(call + ".dR", n * top_k * dx_tiles)
        dx = torch.empty(n, dim, device=grad_out.device, dtype=torch.float32)
        ext().ep_combine(dret[: n * top_k * dim].view(n * top_k, dim), None, top_k, counter, target, dx)
        # Router weights: d w[t, j] = <dY_t, y_(t, j)>, from the rows returned in forward.
        d_weights = (ret_rows.view(n, top_k, dim) * grad_out.unsqueeze(1)).sum(dim=-1)
        return dx, d_weights, None, d_gate, d_up, d_down, None, None


def _static_plan(indices, n_experts, local_experts, capacity, ws):
    """Device-side placement of every assignment into the static slabs:
    (dest_rank, dest_row) int32 (dest_rank -1 = dropped), the keep mask and
    the number of dropped assignments (int32, on the device)."""
    flat_e = indices.reshape(-1)
    within = expert_rank(flat_e, n_experts)  # rank among this expert's assignments
    keep = within < capacity
    slab = ws.world * capacity
    dest_rank = torch.where(keep, torch.div(flat_e, local_experts, rounding_mode="floor"), -1).to(torch.int32)
    dest_row = ((flat_e % local_experts) * slab + ws.rank * capacity + within.clamp(max=capacity - 1)).to(torch.int32)
    dropped = (~keep).sum().to(torch.int32).reshape(1)
    return dest_rank.contiguous(), dest_row.contiguous(), keep, dropped


def _static_slab(ws, key, rows, dim):
    """Static receive slab `key` (rows x dim, zeroed) and its meta (all -1) on
    every rank, created once."""
    fresh = key not in ws._buffers
    buf, ptrs = ws.buffer(key, rows * dim)
    meta_buf, meta_ptrs = ws.buffer(key + ".meta", rows)
    if fresh:
        buf.zero_()
        meta_buf.view(torch.int32).fill_(-1)
        torch.cuda.synchronize(buf.device)
        dist.barrier(group=ws.group)  # every slab is clean before any peer pushes into it
    return buf[: rows * dim].view(rows, dim), ptrs, meta_buf[:rows].view(torch.int32), meta_ptrs


def _static_push(ws, key, src, top_k, dest_rank, dest_row, scale, rows, dim):
    slab, ptrs, meta, meta_ptrs = _static_slab(ws, key, rows, dim)
    off = ws.slots(key)
    epoch = ws.next_epoch(key)
    done = ws._done.get(key)
    if done is None:
        done = ws._done[key] = torch.zeros(1, dtype=torch.int32, device=src.device)
    flags = [p + 4 * (off + ws.rank) for p in ws.signal_ptrs]
    ext().ep_push_rows(src, top_k, dest_rank, dest_row, scale, ptrs, meta_ptrs, flags, ws.rank, epoch, done)
    wait = [ws.signal_ptrs[ws.rank] + 4 * off, 2, epoch, 1, ws.world, ws.rank]
    return slab, meta, wait


class _EPFusedCapacity(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weights, indices, w_gate, w_up, w_down, n_experts, capacity, key):
        ws = tp_fused.workspace(x.device, DIM)
        ws.begin_step()
        call = ws.call_key(key)
        n, dim = x.shape
        top_k = indices.shape[1]
        local_experts = w_gate.shape[0]
        hidden = w_gate.shape[2]
        passes = precision.passes()
        slab_rows = ws.world * capacity
        rows = local_experts * slab_rows
        dest_rank, dest_row, keep, dropped = _static_plan(indices, n_experts, local_experts, capacity, ws)
        xs_all, meta, wait = _static_push(ws, call + ".X", x.contiguous(), top_k, dest_rank, dest_row, None, rows, dim)
        ret, ret_ptrs, counter_ptrs, counter = _return_target(ws, call + ".R", n * top_k, dim)
        n_tiles = ext().gemm_n_tiles(dim, passes)
        # All local experts in one grouped launch per product: the up-projection
        # waits for every rank's pushed rows, the down-projection's epilogue
        # returns each row to its source rank (row map = meta, stacked rows).
        xs3 = xs_all.view(local_experts, slab_rows, dim)
        g = torch.empty(local_experts, slab_rows, hidden, device=x.device, dtype=torch.float32)
        u = torch.empty_like(g)
        h = torch.empty_like(g)
        ext().gemm_swiglu_grouped(xs3, w_gate, w_up, g, u, h, passes, wait)
        scatter = [-1, meta.data_ptr()] + list(ret_ptrs) + list(counter_ptrs)
        ext().gemm_grouped(ret[:dim].view(1, 1, dim), h, [w_down], False, False, _SINGLE, 1.0, False, passes, scatter)
        saved = (g, u, h)
        ext().ep_credit(counter, dropped, n_tiles)
        target = ws.add_target(call + ".R", n * top_k * n_tiles)
        out = torch.empty(n, dim, device=x.device, dtype=torch.float32)
        ret_rows = ret[: n * top_k * dim].view(n * top_k, dim)
        w_kept = (weights.reshape(-1) * keep).contiguous()
        ext().ep_combine(ret_rows, w_kept, top_k, counter, target, out)
        ctx.save_for_backward(weights, w_gate, w_up, w_down, keep, dest_rank, dest_row, dropped)
        ctx.saved = saved
        ctx.meta = (call, n, dim, top_k, hidden, capacity, local_experts)
        ctx.buffers = (xs_all, meta, ret_rows)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        weights, w_gate, w_up, w_down, keep, dest_rank, dest_row, dropped = ctx.saved_tensors
        call, n, dim, top_k, hidden, capacity, local_experts = ctx.meta
        xs_all, meta, ret_rows = ctx.buffers
        ws = tp_fused.workspace(grad_out.device, DIM)
        ws._backward_seen = True
        passes = precision.passes()
        grad_out = grad_out.contiguous()
        slab_rows = ws.world * capacity
        rows = local_experts * slab_rows
        scale = weights.reshape(-1).contiguous()
        dy_all, dy_meta, wait = _static_push(ws, call + ".dY", grad_out, top_k, dest_rank, dest_row, scale, rows, dim)
        dret, dret_ptrs, counter_ptrs, counter = _return_target(ws, call + ".dR", n * top_k, dim)
        d_gate = torch.empty_like(w_gate)
        d_up = torch.empty_like(w_up)
        d_down = torch.empty_like(w_down)
        g, u, h = ctx.saved
        dys3 = dy_all.view(local_experts, slab_rows, dim)
        xs3 = xs_all.view(local_experts, slab_rows, dim)
        dgu = torch.empty(local_experts, slab_rows, 2 * hidden, device=grad_out.device, dtype=torch.float32)
        ext().gemm_swiglu_bwd_grouped(dys3, w_down, g, u, dgu, passes, wait)
        scatter = [-1, meta.data_ptr()] + list(dret_ptrs) + list(counter_ptrs)
        ext().gemm_grouped(dret[:dim].view(1, 1, dim), dgu, [w_gate, w_up], False, True, _SEG_K, 1.0, False, passes,
                           scatter)
        # Unfilled slab rows hold zero gradients (their dY rows are zero), so
        # they add nothing to the weight gradients.
        ext().gemm_grouped(d_gate, xs3, [dgu[..., :hidden]], True, False, _SINGLE, 1.0, False, passes, None)
        ext().gemm_grouped(d_up, xs3, [dgu[..., hidden:]], True, False, _SINGLE, 1.0, False, passes, None)
        ext().gemm_grouped(d_down, h, [dys3], True, False, _SINGLE, 1.0, False, passes, None)
        dx_tiles = ext().gemm_n_tiles(dim, passes)
        ext().ep_credit(counter, dropped, dx_tiles)
        target = ws.add_target(call + ".dR", n * top_k * dx_tiles)
        dx = torch.empty(n, dim, device=grad_out.device, dtype=torch.float32)
        ext().ep_combine(dret[: n * top_k * dim].view(n * top_k, dim), keep.to(torch.float32).contiguous(), top_k,
                         counter, target, dx)
        # This rank's slabs are read for the last time above: clear the meta
        # and the gradient rows its peers filled, before this rank reaches the
        # next step's barrier (after which peers push again).
        meta.fill_(-1)
        dy_all.zero_()
        # Router weights: d w[t, j] = <dY_t, y_(t, j)> for kept slots, 0 for dropped ones.
        d_weights = torch.where(keep.view(n, top_k),
                                (ret_rows.view(n, top_k, dim) * grad_out.unsqueeze(1)).sum(dim=-1),
                                torch.zeros((), device=grad_out.device))
        return dx, d_weights, None, d_gate, d_up, d_down, None, None, None


def dispatch_combine_capacity(x_SD, weights_SK, indices_SK, w_gate_EDM, w_up_EDM, w_down_EMD, n_experts, capacity,
                              key):
    """``dispatch_combine`` with static capacity-bounded slabs (no host sync):
    assignments beyond the first ``capacity`` of their expert on this rank
    (in (token, slot) order) are dropped."""
    return _EPFusedCapacity.apply(x_SD.contiguous(), weights_SK, indices_SK, w_gate_EDM, w_up_EDM, w_down_EMD,
                                  n_experts, int(capacity), key)


def dispatch_combine(x_SD, weights_SK, indices_SK, w_gate_EDM, w_up_EDM, w_down_EMD, n_experts, key):
    """sum_j w[t, j] * expert_{indices[t, j]}(x_t) for this rank's tokens, the
    experts sharded over the "ep" group (``w_*`` are this rank's experts)."""
    return _EPFused.apply(x_SD.contiguous(), weights_SK, indices_SK, w_gate_EDM, w_up_EDM, w_down_EMD, n_experts, key)
