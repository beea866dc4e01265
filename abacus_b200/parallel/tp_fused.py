"""Tensor parallel + Megatron sequence parallel with the collectives fused
into the GEMMs over NVLink peer memory.

Reference semantics: ``abacus/distributed/tensor_parallel.py`` (the SP
all-gather before each column-parallel linear, the reduce-scatter after each
row-parallel linear, mirrored in backward) and ``abacus/attention.py`` /
``abacus/mlp.py`` for the layers. The reference issues each collective as a
separate NCCL call between GEMMs; here:

* all-gather -> GEMM: ``tp_push_rows`` writes this rank's (B, l, D) shard
  into every rank's gathered buffer and publishes an epoch flag; the consuming
  GEMM (QKV, SwiGLU up, or a backward dgrad) reads its local gathered buffer
  and each CTA waits only for the owners of the rows it reads. CTAs over
  this rank's own rows start at once.
* GEMM -> reduce-scatter: the row-parallel GEMM's epilogue stores each
  partial output tile straight into its owner's staging slot over NVLink
  and bumps the owner's arrival counter, so the transfer overlaps the
  remaining tiles' math; ``tp_reduce_rows`` then sums the slots in rank
  order and adds the residual stream in the same pass.

Buffers are symmetric-memory allocations keyed per layer, role and call
within the step (microbatches that run forward before any backward each get
their own), created on first use: every TP rank creates the same keys in the
same order. A bounded device barrier when a new step starts (``begin_step``)
keeps a rank from pushing into a buffer a slower peer may still read from the
previous step's backward.

Requirements (else the NCCL path in ``tensor_parallel`` runs): CUDA fp32,
2..8 ranks, per-rank sequence chunk a multiple of 128 rows.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from abacus_b200.ops import precision
from abacus_b200.ops._ext import ext
from abacus_b200.parallel import mesh

_SIGNAL_INTS = 1 << 16
_BARRIER_SLOTS = 64
_ROW_TILE = 128
_SEG_N, _SEG_K, _SINGLE = 1, 2, 0


def enabled() -> bool:
    return os.environ.get("ABACUS_TP_FUSED", "1") != "0"


def usable(x: torch.Tensor, seq_chunk: int, dim: str = "tp") -> bool:
    """Whether the fused path applies to an SP shard (B, l, D) on the TP group."""
    _, world = mesh.rank_and_world_size(dim)
    return (enabled() and x.is_cuda and x.dtype == torch.float32 and 2 <= world <= 8
            and seq_chunk % _ROW_TILE == 0 and x.shape[-1] % 4 == 0)


class Workspace:
    """Symmetric buffers, flags and counters of one TP group on this rank."""

    def __init__(self, dim: str, device: torch.device):
        from torch.distributed import _symmetric_memory as symm_mem

        self._symm = symm_mem
        self.dim = dim
        self.rank, self.world = mesh.rank_and_world_size(dim)
        group = mesh.group_for(dim)
        self.group = group if group is not None else dist.group.WORLD
        self.device = device
        self.signal, self.signal_ptrs = self._alloc(_SIGNAL_INTS, torch.int32, zero=True)
        self._sig_cursor = _BARRIER_SLOTS
        self._buffers: dict[str, tuple[torch.Tensor, list[int]]] = {}
        self._slots: dict[str, int] = {}
        self._epochs: dict[str, int] = {}
        self._targets: dict[str, int] = {}
        self._done: dict[str, torch.Tensor] = {}
        self._calls: dict[str, int] = {}
        self._backward_seen = False
        self._barrier_epoch = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def _alloc(self, numel: int, dtype, zero: bool = False):
        t = self._symm.empty(numel, dtype=dtype, device=self.device)
        if zero:
            t.zero_()
        handle = self._symm.rendezvous(t, self.group)
        mine = int(handle.buffer_ptrs[self.rank])
        offset = t.data_ptr() - mine
        if offset < 0:
            raise RuntimeError("symmetric tensor lies outside its buffer")
        ptrs = [int(p) + offset for p in handle.buffer_ptrs]
        t._abacus_handle = handle  # keep the mapping alive with the tensor
        return t, ptrs

    # ------------------------------------------------------------------ pieces
    def buffer(self, key: str, numel: int) -> tuple[torch.Tensor, list[int]]:
        entry = self._buffers.get(key)
        if entry is None or entry[0].numel() < numel:
            entry = self._alloc(numel, torch.float32)
            self._buffers[key] = entry
        return entry

    def slots(self, key: str) -> int:
        """Offset of `world` int32 slots (one per source rank) in the signal buffer."""
        off = self._slots.get(key)
        if off is None:
            off = self._sig_cursor
            self._sig_cursor += self.world
            if self._sig_cursor > _SIGNAL_INTS:
                raise RuntimeError("tensor-parallel signal buffer exhausted")
            self._slots[key] = off
        return off

    def next_epoch(self, key: str) -> int:
        e = self._epochs.get(key, 0) + 1
        self._epochs[key] = e
        return e

    def add_target(self, key: str, tiles: int) -> int:
        t = self._targets.get(key, 0) + tiles
        self._targets[key] = t
        return t

    def call_key(self, key: str) -> str:
        """Key of this call of a module since the step began: every microbatch
        of a pipeline step gets its own buffers (backward reuses the key its
        forward saved)."""
        n = self._calls.get(key, 0)
        self._calls[key] = n + 1
        return f"{key}#{n}"

    def begin_step(self, timeout_ms: float = 60_000.0) -> None:
        """Called at every forward. A forward that follows a backward (or runs
        without autograd) starts a new step: call keys restart at 0, so the
        buffers are reused, after a bounded device barrier that every rank
        reaches only once its previous work finished. Further forwards before
        the next backward (microbatches) take fresh keys and need no barrier."""
        if self._calls and not self._backward_seen and torch.is_grad_enabled():
            return
        self._calls.clear()
        self._backward_seen = False
        self._barrier_epoch += 1
        ext().symm_barrier(self.signal_ptrs, self.rank, 0, self._barrier_epoch, timeout_ms, [], None)

    # ------------------------------------------------------------------ collectives
    def push_gather(self, key: str, x2: torch.Tensor, chunk: int, seq: int):
        """Write this rank's (B*l, D) shard into every rank's gathered
        (B*L, D) buffer; returns (local gathered buffer, wait spec)."""
        rows_total = x2.shape[0] * self.world
        buf, ptrs = self.buffer(key, rows_total * x2.shape[1])
        off = self.slots(key)
        epoch = self.next_epoch(key)
        done = self._done.get(key)
        if done is None:
            done = self._done[key] = torch.zeros(1, dtype=torch.int32, device=self.device)
        flag_ptrs = [p + 4 * (off + self.rank) for p in self.signal_ptrs]
        ext().tp_push_rows(x2, ptrs, flag_ptrs, chunk, seq, self.rank, epoch, done)
        wait_flags = self.signal_ptrs[self.rank] + 4 * off
        gathered = buf[: rows_total * x2.shape[1]].view(rows_total, x2.shape[1])
        return gathered, (wait_flags, epoch, chunk, seq, self.rank)

    def scatter_reduce(self, key: str, rows_local: int, n: int, chunk: int, seq: int, launch, residual=None):
        """Run `launch(staging_slot, scatter_spec)` (a GEMM whose epilogue
        scatters rows to their owners; it returns its tiles per owner), then
        reduce the arrived slots (+ residual) into this rank's (rows_local, n)."""
        slot = rows_local * n
        buf, ptrs = self.buffer(key, self.world * slot)
        off = self.slots(key)
        staging = buf[: self.world * slot].view(self.world, rows_local, n)
        scatter = [chunk, seq]
        scatter += [p + 4 * self.rank * slot for p in ptrs]
        scatter += [p + 4 * (off + self.rank) for p in self.signal_ptrs]
        tiles = launch(staging[self.rank], scatter)
        target = self.add_target(key, int(tiles))
        out = torch.empty(rows_local, n, device=self.device, dtype=torch.float32)
        counters = self.signal[off : off + self.world]
        ext().tp_reduce_rows(staging, self.world, counters, target,
                             None if residual is None else residual.contiguous(), out)
        return out


_WORKSPACES: dict = {}


def workspace(device: torch.device, dim: str = "tp") -> Workspace:
    key = (dim, device.index, id(mesh.get_mesh()))
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = _WORKSPACES[key] = Workspace(dim, device)
    return ws


def begin_step(device: torch.device, dim: str = "tp") -> None:
    """Bounded device barrier over the TP group at the start of a forward
    (no-op before the first fused layer created the workspace)."""
    ws = _WORKSPACES.get((dim, device.index, id(mesh.get_mesh())))
    if ws is not None:
        ws.begin_step()


def reset() -> None:
    _WORKSPACES.clear()


def _wait(spec, operand: int) -> list[int]:
    flags, epoch, chunk, seq, rank = spec
    return [flags, operand, epoch, chunk, seq, rank]


def _mm(a, b, trans_a=False, trans_b=False):
    out = torch.empty(a.shape[1] if trans_a else a.shape[0], b.shape[0] if trans_b else b.shape[1],
                      device=a.device, dtype=torch.float32)
    ext().gemm_out(out, a, [b], trans_a, trans_b, _SINGLE, 1.0, None, False, precision.passes())
    return out


# ---------------------------------------------------------------------- layers
class _GatherQKV(torch.autograd.Function):
    """SP shard -> [G @ Wq | G @ Wk | G @ Wv] with G the gathered sequence;
    backward: the dgrad GEMM scatters to the row owners (reduce-scatter)."""

    @staticmethod
    def forward(ctx, x2, wq, wk, wv, key, chunk, seq, dim):
        ws = workspace(x2.device, dim)
        key = ws.call_key(key)
        gathered, spec = ws.push_gather(key + ".G", x2, chunk, seq)
        mats = [w.reshape(w.shape[0], -1) for w in (wq, wk, wv)]
        hk = mats[0].shape[1]
        qkv = torch.empty(gathered.shape[0], 3 * hk, device=x2.device, dtype=torch.float32)
        ext().gemm_out_tp(qkv, gathered, mats, False, False, _SEG_N, 1.0, precision.passes(), _wait(spec, 0), None)
        ctx.save_for_backward(gathered, wq, wk, wv)
        ctx.meta = (key, chunk, seq, dim, x2.shape)
        return qkv

    @staticmethod
    def backward(ctx, dqkv):
        gathered, wq, wk, wv = ctx.saved_tensors
        key, chunk, seq, dim, x_shape = ctx.meta
        ws = workspace(gathered.device, dim)
        ws._backward_seen = True
        dqkv = dqkv.contiguous()
        mats = [w.reshape(w.shape[0], -1) for w in (wq, wk, wv)]
        hk = mats[0].shape[1]
        passes = precision.passes()

        def launch(c, scatter):
            return ext().gemm_out_tp(c, dqkv, mats, False, True, _SEG_K, 1.0, passes, None, scatter)

        dx = ws.scatter_reduce(key + ".dX", x_shape[0], x_shape[1], chunk, seq, launch)
        grads = [_mm(gathered, dqkv[:, i * hk : (i + 1) * hk], trans_a=True).view_as(w)
                 for i, w in enumerate((wq, wk, wv))]
        return (dx, *grads, None, None, None, None)


class _RowScatter(torch.autograd.Function):
    """Row-parallel ``o @ W`` reduce-scattered to the SP shards, plus the
    residual; backward gathers the shard gradient into the dgrad / wgrad GEMMs."""

    @staticmethod
    def forward(ctx, o, w, residual2, key, chunk, seq, dim):
        ws = workspace(o.device, dim)
        key = ws.call_key(key)
        passes = precision.passes()

        def launch(c, scatter):
            return ext().gemm_out_tp(c, o, [w], False, False, _SINGLE, 1.0, passes, None, scatter)

        out = ws.scatter_reduce(key + ".Y", residual2.shape[0], w.shape[1], chunk, seq, launch, residual2)
        ctx.save_for_backward(o, w)
        ctx.meta = (key, chunk, seq, dim)
        return out

    @staticmethod
    def backward(ctx, dout):
        o, w = ctx.saved_tensors
        key, chunk, seq, dim = ctx.meta
        ws = workspace(o.device, dim)
        ws._backward_seen = True
        dout = dout.contiguous()
        gathered, spec = ws.push_gather(key + ".dG", dout, chunk, seq)
        passes = precision.passes()
        do = torch.empty(o.shape, device=o.device, dtype=torch.float32)
        ext().gemm_out_tp(do, gathered, [w], False, True, _SINGLE, 1.0, passes, _wait(spec, 0), None)
        dw = torch.empty(w.shape, device=w.device, dtype=torch.float32)
        ext().gemm_out_tp(dw, o, [gathered], True, False, _SINGLE, 1.0, passes, _wait(spec, 1), None)
        return do, dw, dout, None, None, None, None


class _SwiGLUTP(torch.autograd.Function):
    """SP shard -> gather -> SwiGLU (column-parallel gate/up, row-parallel
    down) -> reduce-scatter + residual, all through the fused paths."""

    @staticmethod
    def forward(ctx, x2, w_gate, w_up, w_down, residual2, key, chunk, seq, dim):
        ws = workspace(x2.device, dim)
        key = ws.call_key(key)
        passes = precision.passes()
        gathered, spec = ws.push_gather(key + ".G", x2, chunk, seq)
        tokens, hidden = gathered.shape[0], w_gate.shape[1]
        g = torch.empty(tokens, hidden, device=x2.device, dtype=torch.float32)
        u = torch.empty_like(g)
        h = torch.empty_like(g)
        ext().gemm_swiglu_tp(gathered, w_gate, w_up, g, u, h, passes, _wait(spec, 0))

        def launch(c, scatter):
            return ext().gemm_out_tp(c, h, [w_down], False, False, _SINGLE, 1.0, passes, None, scatter)

        out = ws.scatter_reduce(key + ".Y", x2.shape[0], w_down.shape[1], chunk, seq, launch, residual2)
        ctx.save_for_backward(gathered, w_gate, w_up, w_down, g, u, h)
        ctx.meta = (key, chunk, seq, dim, x2.shape)
        return out

    @staticmethod
    def backward(ctx, dout):
        gathered, w_gate, w_up, w_down, g, u, h = ctx.saved_tensors
        key, chunk, seq, dim, x_shape = ctx.meta
        ws = workspace(gathered.device, dim)
        ws._backward_seen = True
        passes = precision.passes()
        dout = dout.contiguous()
        hidden = w_gate.shape[1]
        if hidden % 32 != 0:
            raise ValueError("fused TP SwiGLU needs a per-rank hidden size that is a multiple of 32")
        dgath, spec = ws.push_gather(key + ".dG", dout, chunk, seq)
        dgu = torch.empty(dgath.shape[0], 2 * hidden, device=dout.device, dtype=torch.float32)
        ext().gemm_swiglu_bwd_tp(dgath, w_down, g, u, dgu, passes, _wait(spec, 0))

        def launch(c, scatter):
            return ext().gemm_out_tp(c, dgu, [w_gate, w_up], False, True, _SEG_K, 1.0, passes, None, scatter)

        dx = ws.scatter_reduce(key + ".dX", x_shape[0], x_shape[1], chunk, seq, launch)
        grad_wg = _mm(gathered, dgu[:, :hidden], trans_a=True)
        grad_wu = _mm(gathered, dgu[:, hidden:], trans_a=True)
        grad_wd = _mm(h, dgath, trans_a=True)
        return dx, grad_wg, grad_wu, grad_wd, dout, None, None, None, None


_KEYS = {"n": 0}


def new_key(prefix: str) -> str:
    """Per-module key; modules are built in the same order on every rank."""
    _KEYS["n"] += 1
    return f"{prefix}{_KEYS['n']}"


def gather_qkv(x_BlD, wq, wk, wv, key, dim="tp"):
    b, chunk, d = x_BlD.shape
    _, world = mesh.rank_and_world_size(dim)
    return _GatherQKV.apply(x_BlD.reshape(b * chunk, d).contiguous(), wq, wk, wv, key, chunk, chunk * world, dim)


def row_scatter(o, w, residual_BlD, key, dim="tp"):
    b, chunk, d = residual_BlD.shape
    _, world = mesh.rank_and_world_size(dim)
    out = _RowScatter.apply(o.contiguous(), w, residual_BlD.reshape(b * chunk, d), key, chunk, chunk * world, dim)
    return out.view(b, chunk, d)


def swiglu(x_BlD, w_gate, w_up, w_down, residual_BlD, key, dim="tp"):
    b, chunk, d = x_BlD.shape
    _, world = mesh.rank_and_world_size(dim)
    out = _SwiGLUTP.apply(x_BlD.reshape(b * chunk, d).contiguous(), w_gate, w_up, w_down,
                          residual_BlD.reshape(b * chunk, d), key, chunk, chunk * world, dim)
    return out.view(b, chunk, d)
