"""ZeRO-3 / FSDP with its collectives on NVLink peer memory.

Semantics are those of :class:`DataParallel` stage 3
(``abacus/distributed/data_parallel.py:229-345``): parameters, gradients and
Adam moments are sharded over the data-parallel ranks in the reference's
layout (a unit's parameters end to end, cut into equal chunks), each unit
(embedding, every block, final norm, the remaining root parameters) is
gathered for its forward and again for its backward, and the update is one
AdamW step on the token-weighted mean gradient. The reference does each
gather and each gradient reduce-scatter as an NCCL call and steps AdamW after
backward; here:

* parameter all-gather: every rank pushes its chunk of a unit straight into
  every rank's gathered buffer (``tp_push_rows`` over the unit's flat chunk,
  P2P stores) and publishes an epoch flag; the compute stream waits for the W
  flags before the unit runs, and the unit's GEMMs read the gathered buffer
  in place. The next unit's push is issued one unit ahead on a side stream,
  so it overlaps the current unit's compute. Gathered buffers are a pool of
  two symmetric slots (units alternate); a bounded peer barrier before each
  push guarantees that no rank still reads the slot being overwritten.
* gradient reduce-scatter + AdamW: as backward completes a unit, its
  gradients are copied into a pooled symmetric gradient slot, and on the side
  stream a bounded barrier is followed by one kernel (``ar_adamw`` with a
  local slice) in which rank r reads its chunk of every peer's gradient over
  NVLink, forms the token-weighted mean and applies AdamW to the chunk it
  stores -- under the rest of backward. A second barrier frees the slot.

Every device wait is bounded (``timeout_ms``); a wait that runs out sets the
device status word and the fused kernels return without touching memory.
"""
from __future__ import annotations

import itertools

import torch
import torch.distributed as dist

from abacus_b200.ops._ext import ext
from abacus_b200.parallel.data_parallel import DIM, DataParallel
from abacus_b200.utils.fault import PeerFailure

_ROW = 256  # floats per pushed row (the push kernel moves rows of float4s)
_MAX_RANKS = 8
_SLOTS = 2
_SIGNAL_INTS = 4096
_BARRIER_SLOTS = 8
_EXCH = 4
_FLAG_WAIT_MS = 10_000.0  # longest single flag wait the wait kernel accepts


def _round_up(x: int, m: int) -> int:
    return -(-x // m) * m


class _Unit:
    """One unit's parameters in a padded flat space of ``world * chunk``
    floats; this rank owns ``[rank * chunk, (rank + 1) * chunk)``."""

    def __init__(self, index: int, params: list[torch.nn.Parameter], rank: int, world: int):
        self.index = index
        self.params = params
        self.shapes = [tuple(p.shape) for p in params]
        self.sizes = [p.numel() for p in params]
        self.starts = list(itertools.accumulate(self.sizes, initial=0))[:-1]
        self.total = sum(self.sizes)
        self.chunk = _round_up(max(1, -(-self.total // world)), _ROW)
        self.padded = self.chunk * world
        first, last = rank * self.chunk, (rank + 1) * self.chunk
        self.pieces = []  # (lo, hi, at): own flat range of the param inside the chunk
        for start, size in zip(self.starts, self.sizes):
            a, b = max(start, first), min(start + size, last)
            self.pieces.append((a - start, b - start, a - first) if a < b else (0, 0, 0))
        self.index_of = {id(p): i for i, p in enumerate(params)}
        self.local: torch.Tensor | None = None  # this rank's chunk of the values
        self.exp_avg: torch.Tensor | None = None
        self.exp_avg_sq: torch.Tensor | None = None
        self.arrived: set[int] = set()
        self.launched = False
        self.gslot = -1
        self.push_epoch = 0  # epoch of the latest push of this unit

    def piece_views(self, chunk: torch.Tensor) -> list[torch.Tensor]:
        return [chunk[at : at + hi - lo] for lo, hi, at in self.pieces]


class FusedZero3(DataParallel):
    """Stage-3 data parallelism with push all-gathers and a fused
    reduce-scatter + AdamW over NVLink peer memory (CUDA only)."""

    fused_optimizer = True

    def __init__(self, model: torch.nn.Module, dim: str = DIM, token_weighted: bool = True,
                 timeout_ms: float = 60_000.0):
        super().__init__(model, stage=3, dim=dim, token_weighted=token_weighted)
        if self.world_size > _MAX_RANKS:
            raise ValueError(f"fused ZeRO-3 supports at most {_MAX_RANKS} ranks, got {self.world_size}")
        self.timeout_ms = float(timeout_ms)
        self._epoch = 0
        self._stepped = 0
        self._prepared = None
        self._status_host = None
        self._status_event = None

    # ------------------------------------------------------------------ setup
    @torch.no_grad()
    def broadcast_parameters(self) -> None:
        from torch.distributed import _symmetric_memory as symm_mem

        params = [p for p in self._params() if p.requires_grad]
        if not params:
            raise ValueError("model has no trainable parameters")
        device = params[0].device
        if device.type != "cuda" or any(p.dtype != torch.float32 or p.device != device for p in params):
            raise RuntimeError("FusedZero3 needs fp32 CUDA parameters on one device")
        for p in self._params():
            dist.broadcast(p.data, src=self.src, group=self.group)
        for b in self.model.buffers():
            dist.broadcast(b, src=self.src, group=self.group)

        # Units in forward order: embedding, blocks, final norm, then the rest.
        covered, groups, modules = set(), [], []
        for module in self._unit_modules():
            ps = [p for p in module.parameters() if p.requires_grad and id(p) not in covered
                  and id(p) not in self.excluded]
            if ps:
                groups.append(ps)
                modules.append(module)
                covered.update(id(p) for p in ps)
        rest = [p for p in params if id(p) not in covered]
        if rest:
            groups.append(rest)
            modules.append(None)
        self.zunits = [_Unit(i, ps, self.rank, self.world_size) for i, ps in enumerate(groups)]
        self.units = self.zunits  # checkpoint helpers read the units' shapes and pieces
        biggest = max(u.padded for u in self.zunits)

        # Symmetric allocation: gathered slots | gradient slots | signals | exchange rows.
        layout, at = {}, 0
        for name, nbytes in (("gather", _SLOTS * biggest * 4), ("grad", _SLOTS * biggest * 4),
                             ("signal", _SIGNAL_INTS * 4), ("exch", _round_up(_EXCH * self.world_size, 64) * 4)):
            layout[name] = (at, nbytes)
            at = _round_up(at + nbytes, 256)
        raw = symm_mem.empty(at, dtype=torch.uint8, device=device)
        raw.zero_()
        group = self.group if self.group is not None else dist.group.WORLD
        handle = symm_mem.rendezvous(raw, group)
        base = raw.data_ptr() - int(handle.buffer_ptrs[self.rank])
        if base < 0 or base + at > int(handle.buffer_size):
            raise RuntimeError("symmetric buffer does not contain the allocated tensor")

        def view(name, dtype):
            off, nbytes = layout[name]
            return raw[off : off + nbytes].view(dtype)

        def peers(name):
            return [int(p) + base + layout[name][0] for p in handle.buffer_ptrs]

        self._raw, self._handle = raw, handle
        self._biggest = biggest
        self._gather = view("gather", torch.float32).view(_SLOTS, biggest)
        self._grads = view("grad", torch.float32).view(_SLOTS, biggest)
        self._signal = view("signal", torch.int32)
        self._gather_ptrs, self._grad_ptrs = peers("gather"), peers("grad")
        self._signal_ptrs, exch = peers("signal"), peers("exch")
        rows = view("exch", torch.float32)
        self._exch_loss = rows[: 2 * self.world_size].view(self.world_size, 2)
        self._exch_counts = rows[2 * self.world_size : 4 * self.world_size].view(self.world_size, 2)
        self._exch_loss_ptrs = exch
        self._exch_count_ptrs = [p + 8 * self.world_size for p in exch]
        self._done = torch.zeros(len(self.zunits) * _SLOTS, dtype=torch.int32, device=device)
        self._wait_result = torch.zeros(1, dtype=torch.int32, device=device)

        # Local chunks and moments; parameters rest on their local pieces.
        self.owned = {}
        for u in self.zunits:
            u.local = torch.zeros(u.chunk, dtype=torch.float32, device=device)
            u.exp_avg = torch.zeros_like(u.local)
            u.exp_avg_sq = torch.zeros_like(u.local)
            for p, (lo, hi, at_) in zip(u.params, u.pieces):
                if lo < hi:
                    u.local[at_ : at_ + hi - lo].copy_(p.data.reshape(-1)[lo:hi])
                    self.owned[id(p)] = (lo, hi)
            self._to_local(u)
        self.grad_shards = None
        self._unit_of = {id(p): u for u in self.zunits for p in u.params}

        # Hooks: gather before a unit's forward and backward, release after.
        order = self.zunits
        for u, module in zip(order, modules):
            nxt = order[u.index + 1] if u.index + 1 < len(order) else None
            prv = order[u.index - 1] if u.index > 0 else None
            if module is not None:
                module.register_forward_pre_hook(lambda _m, _a, u=u, n=nxt: self._enter(u, n))
                module.register_forward_hook(lambda _m, _a, _o, u=u: self._to_local(u))
                module.register_full_backward_pre_hook(lambda _m, _g, u=u, n=prv: self._enter(u, n))
        if modules and modules[-1] is None:
            root = order[-1]
            last = modules[-2] if len(modules) > 1 else None
            if last is not None:
                last.register_forward_hook(lambda _m, _a, _o, u=root: self._enter(u, None))
            else:
                self.model.register_forward_pre_hook(lambda _m, _a, u=root: self._enter(u, None))
            self.model.register_forward_hook(lambda _m, _a, _o, u=root: self._to_local(u))
            self.model.register_full_backward_pre_hook(
                lambda _m, _g, u=root, n=(order[-2] if len(order) > 1 else None): self._enter(u, n))
        for p in params:
            p.register_post_accumulate_grad_hook(self._on_grad)
        self._comm = torch.cuda.Stream(device=device)
        self._status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._status_event = torch.cuda.Event()
        self._slot_of: dict[int, int] = {}
        self._gslot_free = [None] * _SLOTS
        self._gcount = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    # ------------------------------------------------------------------ gathers
    def _to_local(self, u: _Unit) -> None:
        for p, (lo, hi, at_) in zip(u.params, u.pieces):
            p.data = u.local[at_ : at_ + hi - lo]

    def _barrier(self, exch_ptrs=None, payload=None) -> None:
        self._epoch += 1
        if payload is None:
            ext().symm_barrier(self._signal_ptrs, self.rank, 0, self._epoch, self.timeout_ms, [], None)
        else:
            ext().symm_barrier(self._signal_ptrs, self.rank, 0, self._epoch, self.timeout_ms, exch_ptrs,
                               payload.contiguous())

    def _flag_offset(self, u: _Unit) -> int:
        return _BARRIER_SLOTS + u.index * self.world_size

    def _push(self, u: _Unit) -> None:
        """On the side stream: barrier (the slot is free on every rank), then
        push this rank's chunk of `u` into every rank's gathered slot."""
        slot = self._next_slot(u)
        compute = torch.cuda.current_stream(u.local.device)
        self._comm.wait_stream(compute)
        with torch.cuda.stream(self._comm):
            self._barrier()
            u.push_epoch += 1
            rows = u.chunk // _ROW
            dst = [p + 4 * slot * self._biggest for p in self._gather_ptrs]
            flags = [p + 4 * (self._flag_offset(u) + self.rank) for p in self._signal_ptrs]
            ext().tp_push_rows(u.local.view(rows, _ROW), dst, flags, rows, rows * self.world_size, self.rank,
                               u.push_epoch, self._done[u.index * _SLOTS + slot : u.index * _SLOTS + slot + 1])
            pushed = torch.cuda.Event()
            pushed.record(self._comm)
        self._slot_of[u.index] = (slot, pushed)

    def _next_slot(self, u: _Unit) -> int:
        return u.index % _SLOTS

    def _enter(self, u: _Unit, upcoming: _Unit | None) -> None:
        with torch.no_grad():
            if self._slot_of.get(u.index) is None:
                self._push(u)
            # The compute stream orders itself after this rank's own push (an
            # event: no kernel of this GPU spins on another of its kernels)
            # and waits, bounded, for every peer's chunk flag.
            slot, pushed = self._slot_of.pop(u.index)
            compute = torch.cuda.current_stream(u.local.device)
            compute.wait_event(pushed)
            off = self._flag_offset(u)
            for r in range(self.world_size):
                if r != self.rank:
                    ext().wait_flag(self._signal[off + r : off + r + 1], u.push_epoch,
                                    min(self.timeout_ms, _FLAG_WAIT_MS), self._wait_result)
            flat = self._gather[slot, : u.padded]
            for p, s, n, shape in zip(u.params, u.starts, u.sizes, u.shapes):
                p.data = flat[s : s + n].view(shape)
            if upcoming is not None and self._slot_of.get(upcoming.index) is None:
                self._push(upcoming)

    # ------------------------------------------------------------------ step
    def set_token_count(self, token_count) -> None:
        self._token_count = token_count
        for u in self.zunits:
            u.arrived.clear()
            u.launched = False
            u.gslot = -1

    @torch.no_grad()
    def prepare_step(self, optimizer, token_count) -> None:
        """This step's AdamW hyper-parameters and token count, before backward."""
        self._check_previous()
        self._stepped += 1
        for p in optimizer.params:
            st = optimizer.state.get(id(p))
            if st is not None:
                st["step"] = self._stepped
        self._prepared = (float(optimizer.lr), optimizer.beta1, optimizer.beta2, optimizer.eps,
                          optimizer.weight_decay, self._stepped)
        self.set_token_count(token_count)
        device = self.zunits[0].local.device
        if self.token_weighted:
            count = torch.as_tensor(token_count, device=device).reshape(()).to(torch.float32)
        else:
            count = torch.ones((), device=device, dtype=torch.float32)
        self._count_payload = torch.stack((count, torch.zeros_like(count)))
        self._counts_sent = False

    @torch.no_grad()
    def _on_grad(self, p) -> None:
        u = self._unit_of[id(p)]
        i = u.index_of[id(p)]
        if i in u.arrived:
            raise RuntimeError(f"a {tuple(p.shape)} parameter received a second gradient in one backward")
        if u.gslot < 0:
            self._open_grad_slot(u)
        s, n = u.starts[i], u.sizes[i]
        self._grads[u.gslot, s : s + n].copy_(p.grad.reshape(-1))
        p.grad = None
        u.arrived.add(i)
        if len(u.arrived) == len(u.params) and self._prepared is not None:
            self._to_local(u)  # backward is done with the gathered values
            self._reduce(u)

    def _open_grad_slot(self, u: _Unit) -> None:
        slot = self._gcount % _SLOTS
        self._gcount += 1
        free = self._gslot_free[slot]
        if free is not None:
            torch.cuda.current_stream(u.local.device).wait_event(free)
        u.gslot = slot
        # The slot's padding tail must read as zero gradients.
        self._grads[slot, u.total : u.padded].zero_()

    def _reduce(self, u: _Unit) -> None:
        """Side stream: barrier (every rank's gradients of u are in place),
        reduce-scatter + AdamW into the local chunk, barrier (slot free)."""
        compute = torch.cuda.current_stream(u.local.device)
        self._comm.wait_stream(compute)
        lr, beta1, beta2, eps, wd, step = self._prepared
        with torch.cuda.stream(self._comm):
            if not self._counts_sent:
                self._barrier(self._exch_count_ptrs, self._count_payload)
                self._counts_sent = True
            else:
                self._barrier()
            lo = self.rank * u.chunk
            grads = [p + 4 * u.gslot * self._biggest for p in self._grad_ptrs]
            ext().ar_adamw(grads, [0] * self.world_size, self._exch_counts[:, 0], self.token_weighted, self.rank,
                           lo, lo + u.chunk, u.exp_avg, u.exp_avg_sq, lr, beta1, beta2, eps, wd, step, 0, u.local)
            self._barrier()
            ev = torch.cuda.Event()
            ev.record(self._comm)
            self._gslot_free[u.gslot] = ev
        u.launched = True

    @torch.no_grad()
    def synchronize(self, loss: torch.Tensor, token_count) -> torch.Tensor:
        if self._prepared is None:
            raise RuntimeError("FusedZero3.prepare_step must run before backward")
        for u in self.zunits:
            if not u.launched:
                if u.gslot < 0:
                    self._open_grad_slot(u)
                for i in range(len(u.params)):
                    if i not in u.arrived:
                        s, n = u.starts[i], u.sizes[i]
                        self._grads[u.gslot, s : s + n].zero_()
                        u.arrived.add(i)
                self._reduce(u)
        loss32 = loss.detach().reshape(()).to(torch.float32)
        if self.token_weighted:
            count = torch.as_tensor(token_count, device=loss32.device).reshape(()).to(torch.float32)
            payload = torch.stack((loss32 * count, count))
        else:
            payload = torch.stack((loss32, torch.ones_like(loss32)))
        compute = torch.cuda.current_stream(loss32.device)
        self._comm.wait_stream(compute)
        with torch.cuda.stream(self._comm):
            self._barrier(self._exch_loss_ptrs, payload)
        compute.wait_stream(self._comm)
        payload.record_stream(self._comm)
        self._count_payload.record_stream(self._comm)
        rows = self._exch_loss
        mean = rows[:, 0].sum() / rows[:, 1].sum() if self.token_weighted else rows[:, 0].sum()
        self._prepared = None
        self._gslot_free = [None] * _SLOTS
        self._gcount = 0
        self._status_host.copy_(ext().status_tensor(loss32.device.index), non_blocking=True)
        self._status_event.record()
        return mean.to(loss.dtype)

    def step_optimizer(self, optimizer) -> None:
        return

    def bind_optimizer(self, optimizer) -> None:
        """Moments live in the units' chunks; the optimizer's per-parameter
        state views them (for checkpoints)."""
        for u in self.zunits:
            for p, (lo, hi, at_) in zip(u.params, u.pieces):
                if lo < hi:
                    optimizer.state[id(p)] = {"step": self._stepped, "exp_avg": u.exp_avg[at_ : at_ + hi - lo],
                                              "exp_avg_sq": u.exp_avg_sq[at_ : at_ + hi - lo]}

    def gather_parameters(self) -> None:
        return

    @torch.no_grad()
    def gather_owned(self, pieces: dict[int, torch.Tensor]) -> dict[int, torch.Tensor]:
        """Full flattened tensors from every rank's owned pieces (collective)."""
        out = {}
        for u in self.zunits:
            chunk = torch.zeros_like(u.local)
            for p, view in zip(u.params, u.piece_views(chunk)):
                src = pieces.get(id(p))
                if src is not None and view.numel():
                    view.copy_(src.reshape(-1))
            flat = self._gather_chunks(chunk)
            for p, s, n in zip(u.params, u.starts, u.sizes):
                out[id(p)] = flat[s : s + n].clone()
        return out

    @torch.no_grad()
    def full_parameters(self) -> list[torch.Tensor]:
        full = {}
        for u in self.zunits:
            flat = self._gather_chunks(u.local)
            for p, s, n, shape in zip(u.params, u.starts, u.sizes, u.shapes):
                full[id(p)] = flat[s : s + n].view(shape).clone()
        return [full.get(id(p), p.detach().clone()) for p in self.model.parameters()]

    # ------------------------------------------------------------------ health
    def _check_previous(self) -> None:
        if self._status_event is not None and self._status_event.query():
            self._raise_if_failed(int(self._status_host[0]))

    def _raise_if_failed(self, code: int) -> None:
        if code != 0:
            raise PeerFailure(f"fused ZeRO-3 step on rank {self.rank} reported device status {code} "
                              "(a peer did not arrive within the wait limit)")

    def check(self) -> None:
        if self._status_event is not None:
            self._status_event.synchronize()
            self._raise_if_failed(int(self._status_host[0]))

    def release(self) -> None:
        torch.cuda.synchronize(self.zunits[0].local.device)
        for u in self.zunits:
            for p in u.params:
                p.data = p.data.clone()
        self._raw = self._handle = None
