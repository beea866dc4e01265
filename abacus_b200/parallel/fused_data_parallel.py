"""DDP whose gradient all-reduce and AdamW step are one NVLink kernel.

Semantics are those of :class:`DataParallel` stage 0 followed by
:class:`AdamW` (``abacus/distributed/data_parallel.py:141-161`` token-weighted
mean gradient, ``abacus/optimizers/adamw.py`` update): after a step every
replica holds the same parameters, equal to one AdamW step on
``sum_r count_r * g_r / sum_r count_r``.

Layout. All trainable parameters live in one flat fp32 buffer allocated in
symmetric memory (``torch.distributed._symmetric_memory``): every rank maps
every peer's buffer, so a kernel can load and store a peer's memory over
NVLink. Each parameter starts on a 16-byte boundary (TMA-aligned views).
Gradients are copied by a post-accumulate hook into a second flat buffer in
the same allocation, and the autograd gradient is released at once, so no
gradient outlives backward outside that buffer. The flat range is split
evenly (in float4 units) between ranks; rank r keeps the Adam moments of its
slice only (ZeRO-1 sized optimizer state).

One step (``synchronize`` then ``step_optimizer``), all on the current stream:

1. ``symm_barrier`` with payload: every rank's gradients are complete, and the
   pair (loss * count, count) of every rank lands in each rank's exchange
   rows. The global mean loss is computed from those rows; no NCCL call.
2. ``ar_adamw``: rank r reads its slice of every peer's gradient over NVLink,
   forms the token-weighted mean, applies AdamW, and writes the new values into
   every peer's parameter buffer: reduce-scatter + optimizer + all-gather in
   one pass over the slice.
3. ``symm_barrier``: every peer's stores have landed and every peer is done
   reading this rank's gradients before the next backward overwrites them.

Every device-side wait is bounded (``timeout_ms``); a wait that runs out
sets the device status word, the fused kernels then return without touching
memory, and the next ``step_optimizer`` (or ``check``) raises ``PeerFailure``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from abacus_b200.ops._ext import ext
from abacus_b200.parallel.data_parallel import DIM, DataParallel
from abacus_b200.utils.fault import PeerFailure

_ALIGN = 4  # float4: 16 bytes
_MAX_RANKS = 8
_SIGNAL_SLOTS = 64


def _round_up(x: int, m: int) -> int:
    return -(-x // m) * m


class FusedDataParallel(DataParallel):
    """Stage-0 data parallelism fused with AdamW over NVLink peer memory (CUDA only)."""

    fused_optimizer = True

    def __init__(self, model: torch.nn.Module, dim: str = DIM, token_weighted: bool = True,
                 timeout_ms: float = 60_000.0):
        super().__init__(model, stage=0, dim=dim, token_weighted=token_weighted)
        if self.world_size > _MAX_RANKS:
            raise ValueError(f"fused data parallel supports at most {_MAX_RANKS} ranks, got {self.world_size}")
        self.timeout_ms = float(timeout_ms)
        self._flat_params: list[torch.nn.Parameter] = []
        self._epoch = 0
        self._ready: set[int] = set()
        self._status_host = None
        self._status_event = None
        self._mean = None
        self._stepped = 0

    # ------------------------------------------------------------------ setup
    @torch.no_grad()
    def broadcast_parameters(self) -> None:
        from torch.distributed import _symmetric_memory as symm_mem

        params = [p for p in self._params() if p.requires_grad]
        if not params:
            raise ValueError("model has no trainable parameters")
        device = params[0].device
        if device.type != "cuda":
            raise RuntimeError("FusedDataParallel needs CUDA parameters (NVLink peer memory)")
        if any(p.dtype != torch.float32 or p.device != device for p in params):
            raise RuntimeError("FusedDataParallel needs fp32 parameters on one device")
        for p in self._params():
            dist.broadcast(p.data, src=self.src, group=self.group)
        for b in self.model.buffers():
            dist.broadcast(b, src=self.src, group=self.group)

        offsets, total = [], 0
        for p in params:
            offsets.append(total)
            total = _round_up(total + p.numel(), _ALIGN)
        padded = _round_up(max(total, 1), _ALIGN * self.world_size)
        shard = padded // self.world_size
        self._lo, self._hi = self.rank * shard, (self.rank + 1) * shard

        # One symmetric allocation: params | grads | signal slots | exchange rows.
        exch_floats = _round_up(2 * self.world_size, 64)
        layout = {}
        cursor = 0
        for name, nbytes in (("param", padded * 4), ("grad", padded * 4), ("signal", _SIGNAL_SLOTS * 4),
                             ("exch", exch_floats * 4)):
            layout[name] = (cursor, nbytes)
            cursor = _round_up(cursor + nbytes, 256)
        raw = symm_mem.empty(cursor, dtype=torch.uint8, device=device)
        raw.zero_()
        group = self.group if self.group is not None else dist.group.WORLD
        handle = symm_mem.rendezvous(raw, group)
        mine = int(handle.buffer_ptrs[self.rank])
        base = raw.data_ptr() - mine
        if base < 0 or base + cursor > int(handle.buffer_size):
            raise RuntimeError("symmetric buffer does not contain the allocated tensor")

        def view(name, dtype):
            off, nbytes = layout[name]
            return raw[off : off + nbytes].view(dtype)

        def peers(name):
            off = layout[name][0]
            return [int(ptr) + base + off for ptr in handle.buffer_ptrs]

        self._raw, self._handle = raw, handle
        self._param_flat = view("param", torch.float32)
        self._grad_flat = view("grad", torch.float32)
        self._exch = view("exch", torch.float32)[: 2 * self.world_size].view(self.world_size, 2)
        self._param_ptrs, self._grad_ptrs = peers("param"), peers("grad")
        self._signal_ptrs, self._exch_ptrs = peers("signal"), peers("exch")

        for p, off in zip(params, offsets):
            n = p.numel()
            self._param_flat[off : off + n].copy_(p.data.reshape(-1))
            p.data = self._param_flat[off : off + n].view(p.shape)
        self._flat_params = params
        self._offsets = offsets
        self._index = {id(p): i for i, p in enumerate(params)}

        # Moments of the owned slice, and per-parameter views of them (the
        # optimizer state, ZeRO-1 style: exp_avg of the owned flat range).
        self._exp_avg = torch.zeros(shard, dtype=torch.float32, device=device)
        self._exp_avg_sq = torch.zeros(shard, dtype=torch.float32, device=device)
        self.owned = {}
        self._moment_views = {}
        for p, off in zip(params, offsets):
            begin, stop = max(0, self._lo - off), min(p.numel(), self._hi - off)
            if begin < stop:
                self.owned[id(p)] = (begin, stop)
                dest = off + begin - self._lo
                self._moment_views[id(p)] = (self._exp_avg[dest : dest + stop - begin],
                                             self._exp_avg_sq[dest : dest + stop - begin])
        self.grad_shards = None
        for p in params:
            p.register_post_accumulate_grad_hook(self._on_grad_fused)
        self._status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._status_event = torch.cuda.Event()
        # Every rank's zeroed buffer is in place before any peer writes to it.
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    # ------------------------------------------------------------------ backward
    def set_token_count(self, token_count) -> None:
        self._token_count = token_count
        self._ready.clear()

    @torch.no_grad()
    def _on_grad_fused(self, p):
        i = self._index[id(p)]
        off = self._offsets[i]
        self._grad_flat[off : off + p.numel()].copy_(p.grad.reshape(-1))
        self._ready.add(i)
        p.grad = None

    @torch.no_grad()
    def synchronize(self, loss: torch.Tensor, token_count) -> torch.Tensor:
        """Barrier 1 (gradients complete, counts exchanged); returns the global mean loss."""
        self._check_previous()
        if not self._ready:
            raise RuntimeError("backward produced no gradients")
        for i, p in enumerate(self._flat_params):
            if i not in self._ready:
                off = self._offsets[i]
                self._grad_flat[off : off + p.numel()].zero_()
        loss32 = loss.detach().reshape(()).to(torch.float32)
        if self.token_weighted:
            count = torch.as_tensor(token_count, device=loss32.device).reshape(()).to(torch.float32)
            payload = torch.stack((loss32 * count, count))
        else:
            payload = torch.stack((loss32, torch.ones_like(loss32)))
        self._barrier(payload)
        if self.token_weighted:
            mean = self._exch[:, 0].sum() / self._exch[:, 1].sum()
        else:
            mean = self._exch[:, 0].sum()
        self._mean = mean.to(loss.dtype)
        return self._mean

    # ------------------------------------------------------------------ optimizer
    @torch.no_grad()
    def step_optimizer(self, optimizer) -> None:
        """Fused reduce + AdamW + parameter broadcast, then barrier 2."""
        if self._mean is None:
            raise RuntimeError("step_optimizer must follow synchronize")
        self._mean = None
        self._adopt_state(optimizer)
        step = 0
        for p in self._flat_params:
            st = optimizer.state.get(id(p))
            if st is not None:
                st["step"] += 1
                step = max(step, int(st["step"]))
        step = max(step, self._stepped + 1)
        self._stepped = step
        ext().ar_adamw(
            self._grad_ptrs, self._param_ptrs, self._exch[:, 1], self.token_weighted, self.rank, self._lo, self._hi,
            self._exp_avg, self._exp_avg_sq, float(optimizer.lr), optimizer.beta1, optimizer.beta2, optimizer.eps,
            optimizer.weight_decay, step,
        )
        self._barrier(None)
        self._status_host.copy_(ext().status_tensor(self._grad_flat.device.index), non_blocking=True)
        self._status_event.record()

    def _adopt_state(self, optimizer) -> None:
        """Point the optimizer's state at the flat moment slices (copying in any
        state that was loaded from a checkpoint since the last step)."""
        for p in self._flat_params:
            views = self._moment_views.get(id(p))
            if views is None:
                continue
            st = optimizer.state.get(id(p))
            if st is None:
                st = optimizer.state[id(p)] = {"step": self._stepped, "exp_avg": views[0], "exp_avg_sq": views[1]}
            for key, v in zip(("exp_avg", "exp_avg_sq"), views):
                if st[key] is not v:
                    if st[key].data_ptr() != v.data_ptr():
                        v.copy_(st[key].reshape(-1))
                    st[key] = v

    def bind_optimizer(self, optimizer) -> None:
        self._adopt_state(optimizer)

    # ------------------------------------------------------------------ health
    def _barrier(self, payload) -> None:
        self._epoch += 1
        if payload is None:
            ext().symm_barrier(self._signal_ptrs, self.rank, 0, self._epoch, self.timeout_ms, [], None)
        else:
            ext().symm_barrier(self._signal_ptrs, self.rank, 0, self._epoch, self.timeout_ms, self._exch_ptrs,
                               payload.contiguous())

    def _check_previous(self) -> None:
        if self._status_event is not None and self._status_event.query():
            self._raise_if_failed(int(self._status_host[0]))

    def _raise_if_failed(self, code: int) -> None:
        if code != 0:
            raise PeerFailure(f"fused data-parallel step on rank {self.rank} reported device status {code} "
                              "(a peer did not arrive within the wait limit)")

    def check(self) -> None:
        """Wait for the last step and raise ``PeerFailure`` if a device wait ran out."""
        if self._status_event is not None:
            self._status_event.synchronize()
            self._raise_if_failed(int(self._status_host[0]))

    def gather_parameters(self) -> None:
        return

    def release(self) -> None:
        """Drop the symmetric buffers (parameters are copied back to private memory)."""
        for p in self._flat_params:
            p.data = p.data.clone()
        self._flat_params = []
        self._raw = self._handle = None
