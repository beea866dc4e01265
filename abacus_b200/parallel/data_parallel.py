"""Data parallelism: DDP (ZeRO-0) and ZeRO-1/2/3, token-weighted.

API and semantics follow ``abacus/distributed/data_parallel.py``: gradients
are the token-weighted mean over every rank's targets (each rank's gradient is
multiplied by its local target count, summed over ranks, divided by the global
count); stage 1 shards the Adam moments, stage 2 also the gradients, stage 3
also the parameters. ``owned`` (``id(param) -> (begin, end)`` of the flattened
parameter) and ``grad_shards`` feed the ZeRO-aware AdamW, and the sharding
layout is the reference's: a unit's parameters laid end to end, cut into
``world`` equal chunks with the tail of the last one padded.

Design (B200-first, NCCL collectives on the "dp" group of the installed mesh):

* Stage 0: gradients are packed into ~25 MB buckets by post-accumulate hooks
  and each bucket's all-reduce starts asynchronously while backward continues.
  Buckets launch strictly in index order on every rank, so the NCCL call
  sequence is identical across ranks even when a parameter gets no gradient.
* Every ZeRO unit (:class:`_FlatUnit`) owns flat storage. Stages 1 / 2 keep
  all parameters as views of one padded flat buffer, so the parameter
  all-gather after the optimizer step is one in-place ``all_gather_into_tensor``
  with no packing. Stage 3 keeps this rank's chunk of each unit as one
  contiguous tensor whose pieces are the parameters' storage; a gather reads
  the chunk directly.
* Gradients of every stage are copied into the unit's flat gradient buffer as
  they arrive (post-accumulate hooks) and the autograd gradient is released at
  once. In stage 3 each unit's reduce-scatter starts asynchronously as soon as
  its last gradient arrives, so it overlaps the rest of backward; the next
  unit's parameter all-gather is prefetched one unit ahead in forward and in
  backward.
* The loss / token-count reduction is one 2-element all-reduce.
* Parameters listed in ``exclude`` (e.g. expert weights sharded over the same
  ranks) are neither broadcast nor reduced.
"""
from __future__ import annotations

import itertools

import torch
import torch.distributed as dist

from abacus_b200.parallel import mesh

DIM = "dp"


def _has_parameters(module: torch.nn.Module) -> bool:
    return next(module.parameters(), None) is not None


class _FlatUnit:
    """One ZeRO unit: parameters in a flat index space cut into equal chunks.

    Parameter i covers ``[starts[i], starts[i] + sizes[i])`` of a space of
    ``total`` elements. The space is padded to ``padded = world * chunk`` and
    rank r owns ``[r * chunk, (r + 1) * chunk)``. ``pieces[i] = (lo, hi, at)``:
    elements ``[lo, hi)`` of parameter i's own flattened index lie in this
    rank's chunk, starting at offset ``at`` of the chunk (``lo == hi``: none).
    """

    def __init__(self, params: list[torch.nn.Parameter], rank: int, world: int):
        if not params:
            raise ValueError("a ZeRO unit needs at least one parameter")
        self.params = list(params)
        self.shapes = [tuple(p.shape) for p in self.params]
        self.sizes = [p.numel() for p in self.params]
        self.starts = list(itertools.accumulate(self.sizes, initial=0))[:-1]
        self.total = sum(self.sizes)
        self.world = world
        self.chunk = -(-self.total // world)
        self.padded = self.chunk * world
        first, last = rank * self.chunk, (rank + 1) * self.chunk
        self.pieces: list[tuple[int, int, int]] = []
        for start, size in zip(self.starts, self.sizes):
            a, b = max(start, first), min(start + size, last)
            self.pieces.append((a - start, b - start, a - first) if a < b else (0, 0, 0))
        self.index = {id(p): i for i, p in enumerate(self.params)}
        # Stage-3 parameter state.
        self.local: torch.Tensor | None = None  # this rank's chunk of the values
        self.full: torch.Tensor | None = None  # gathered values while materialised
        self.gathering = None  # in-flight all-gather work
        # Gradient state (every stage).
        self.grad_flat: torch.Tensor | None = None
        self.grad_chunk: torch.Tensor | None = None
        self.arrived: set[int] = set()
        self.scatter = None  # in-flight reduce-scatter work
        self.reduced = False

    def owned(self) -> dict[int, tuple[int, int]]:
        return {id(p): (lo, hi) for p, (lo, hi, _) in zip(self.params, self.pieces) if lo < hi}

    def piece_views(self, chunk: torch.Tensor) -> list[torch.Tensor]:
        """This rank's piece of each parameter inside ``chunk`` (empty if none)."""
        return [chunk[at : at + hi - lo] for lo, hi, at in self.pieces]

    def param_views(self, flat: torch.Tensor) -> list[torch.Tensor]:
        """Each parameter, shaped, inside a full flat buffer of the unit."""
        return [flat[s : s + n].view(shape) for s, n, shape in zip(self.starts, self.sizes, self.shapes)]

    def new_grad_flat(self) -> torch.Tensor:
        p = self.params[0]
        return torch.zeros(self.padded, dtype=p.dtype, device=p.device)

    def reset(self) -> None:
        self.arrived.clear()
        self.reduced = False


class _Bucket:
    def __init__(self, params, device, dtype):
        self.params = params
        self.offsets = []
        total = 0
        for p in params:
            self.offsets.append(total)
            total += p.numel()
        self.flat = torch.zeros(total, device=device, dtype=dtype)
        self.ready: set[int] = set()
        self.work = None
        self.launched = False


class DataParallel:
    """Replica of one model per rank. Gradients are the mean over every rank's tokens."""

    def __init__(
        self,
        model: torch.nn.Module,
        stage: int = 0,
        bucket_mb: float = 25.0,
        exclude=None,
        dim: str = DIM,
        token_weighted: bool = True,
        prefetch: bool = True,
    ):
        if not dist.is_initialized():
            raise RuntimeError("DataParallel needs an initialised process group (call init_process_group first)")
        if stage not in (0, 1, 2, 3):
            raise ValueError(f"ZeRO stage {stage!r} is not one of 0, 1, 2, 3")
        self.model = model
        self.stage = stage
        self.dim = dim
        self.group = mesh.group_for(dim)
        self.rank, self.world_size = mesh.rank_and_world_size(dim)
        self.src = mesh.global_rank(dim, 0)
        self.bucket_bytes = int(bucket_mb * 1024 * 1024)
        self.excluded = {id(p) for p in (exclude or [])}
        # token_weighted: each rank's loss is its local mean, gradients are
        # combined as sum(count_r * g_r) / sum(count_r) (the reference).
        # Otherwise each rank's loss is already divided by the global count and
        # gradients are plain sums (used when expert weights receive every
        # rank's tokens through the expert-parallel all-to-all).
        self.token_weighted = token_weighted
        self.prefetch = prefetch
        self.units: list[_FlatUnit] = []
        self.owned: dict[int, tuple[int, int]] | None = None
        self.grad_shards: dict[int, torch.Tensor] | None = None
        self._token_count = 0
        self._buckets: list[_Bucket] = []
        self._bucket_of: dict[int, tuple[int, int]] = {}
        self._next_launch = 0
        self._hooks_installed = False
        self._flat_params: torch.Tensor | None = None  # stages 1 / 2

    # ------------------------------------------------------------------ helpers
    def _params(self):
        return [p for p in self.model.parameters() if id(p) not in self.excluded]

    def _all_reduce(self, t, async_op=False):
        return dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group, async_op=async_op)

    def _multiplier(self):
        return self._token_count if self.token_weighted else 1.0

    def _scale(self, t: torch.Tensor) -> None:
        count = self._multiplier()
        if isinstance(count, torch.Tensor):
            t.mul_(count.to(t.dtype))
        elif count != 1.0:
            t.mul_(float(count))

    # ------------------------------------------------------------------ API
    def set_token_count(self, token_count) -> None:
        """This rank's target-token count for the coming backward (int or 0-d tensor)."""
        self._token_count = token_count
        for unit in self.units:
            unit.reset()
        for b in self._buckets:
            b.ready.clear()
            b.work = None
            b.launched = False
        self._next_launch = 0

    @torch.no_grad()
    def broadcast_parameters(self) -> None:
        for p in self._params():
            dist.broadcast(p.data, src=self.src, group=self.group)
        for b in self.model.buffers():
            dist.broadcast(b, src=self.src, group=self.group)
        if self.stage == 0:
            self._install_buckets()
            return
        if self.stage == 3:
            self._install_stage3()
        else:
            self._install_flat()
        self.owned = {}
        for unit in self.units:
            self.owned.update(unit.owned())
        self.grad_shards = {} if self.stage >= 2 else None

    @torch.no_grad()
    def synchronize(self, loss: torch.Tensor, token_count) -> torch.Tensor:
        """Reduce gradients after backward; returns the global token-weighted mean loss."""
        mean, total = self._mean_loss(loss, token_count)
        if self.stage == 0:
            self._finish_buckets(total)
        else:
            self._finish_units(total)
        return mean

    @torch.no_grad()
    def gather_parameters(self) -> None:
        """Stages 1 / 2: every rank's updated chunk to every rank, in place."""
        if self.stage not in (1, 2):
            return
        unit = self.units[0]
        mine = self._flat_params[self.rank * unit.chunk : (self.rank + 1) * unit.chunk]
        dist.all_gather_into_tensor(self._flat_params, mine, group=self.group)

    @torch.no_grad()
    def full_parameters(self) -> list[torch.Tensor]:
        if self.stage < 3:
            return [p.detach().clone() for p in self.model.parameters()]
        full = {}
        for unit in self.units:
            flat = self._gather_chunks(unit.local)
            for p, view in zip(unit.params, unit.param_views(flat)):
                full[id(p)] = view.clone()
        return [full.get(id(p), p.detach().clone()) for p in self.model.parameters()]

    @torch.no_grad()
    def gather_owned(self, pieces: dict[int, torch.Tensor]) -> dict[int, torch.Tensor]:
        """Full flattened tensors from per-rank owned pieces (collective).

        ``pieces`` maps ``id(param)`` to this rank's owned range of a per-element
        quantity of that parameter (e.g. an Adam moment); the result maps every
        parameter of the ZeRO units to its full flattened tensor.
        """
        out = {}
        for unit in self.units:
            p0 = unit.params[0]
            chunk = torch.zeros(unit.chunk, dtype=p0.dtype, device=p0.device)
            for p, view in zip(unit.params, unit.piece_views(chunk)):
                src = pieces.get(id(p))
                if src is not None and view.numel():
                    view.copy_(src.reshape(-1))
            flat = self._gather_chunks(chunk)
            for p, s, n in zip(unit.params, unit.starts, unit.sizes):
                out[id(p)] = flat[s : s + n].clone()
        return out

    def _gather_chunks(self, chunk: torch.Tensor) -> torch.Tensor:
        flat = chunk.new_empty(chunk.numel() * self.world_size)
        dist.all_gather_into_tensor(flat, chunk.contiguous(), group=self.group)
        return flat

    # ------------------------------------------------------------------ loss
    def _mean_loss(self, loss, token_count):
        if not self.token_weighted:
            packed = loss.detach().reshape(1).clone()
            self._all_reduce(packed)
            return packed[0], torch.ones((), dtype=loss.dtype, device=loss.device)
        count = torch.as_tensor(token_count, dtype=loss.dtype, device=loss.device).reshape(())
        packed = torch.stack((loss.detach().reshape(()) * count, count))
        self._all_reduce(packed)
        total = packed[1]
        if not loss.is_cuda and total.item() == 0:
            raise RuntimeError("no rank had a target token in this batch")
        return packed[0] / total, total

    # ------------------------------------------------------------------ stage 0
    def _install_buckets(self):
        if self._hooks_installed:
            return
        params = [p for p in self._params() if p.requires_grad]
        # Backward produces gradients roughly in reverse registration order.
        params = list(reversed(params))
        current, size = [], 0
        for p in params:
            nbytes = p.numel() * p.element_size()
            if current and size + nbytes > self.bucket_bytes:
                self._buckets.append(_Bucket(current, p.device, p.dtype))
                current, size = [], 0
            current.append(p)
            size += nbytes
        if current:
            self._buckets.append(_Bucket(current, current[0].device, current[0].dtype))
        for bi, bucket in enumerate(self._buckets):
            for pi, p in enumerate(bucket.params):
                self._bucket_of[id(p)] = (bi, pi)
                p.register_post_accumulate_grad_hook(self._on_grad_stage0)
        self._hooks_installed = True

    @torch.no_grad()
    def _on_grad_stage0(self, p):
        bi, pi = self._bucket_of[id(p)]
        bucket = self._buckets[bi]
        if pi in bucket.ready:
            return
        view = bucket.flat[bucket.offsets[pi] : bucket.offsets[pi] + p.numel()]
        view.copy_(p.grad.reshape(-1))
        bucket.ready.add(pi)
        self._launch_ready()

    def _launch(self, bucket):
        self._scale(bucket.flat)
        bucket.work = self._all_reduce(bucket.flat, async_op=True)
        bucket.launched = True

    def _launch_ready(self):
        while self._next_launch < len(self._buckets):
            bucket = self._buckets[self._next_launch]
            if len(bucket.ready) != len(bucket.params):
                return
            self._launch(bucket)
            self._next_launch += 1

    def _finish_buckets(self, total):
        any_grad = False
        for bucket in self._buckets:
            missing = [pi for pi in range(len(bucket.params)) if pi not in bucket.ready]
            for pi in missing:
                bucket.flat[bucket.offsets[pi] : bucket.offsets[pi] + bucket.params[pi].numel()].zero_()
            any_grad = any_grad or len(missing) < len(bucket.params)
        if self._buckets and not any_grad:
            raise RuntimeError("backward produced no gradients")
        while self._next_launch < len(self._buckets):
            self._launch(self._buckets[self._next_launch])
            self._next_launch += 1
        inv = 1.0 / total
        for bucket in self._buckets:
            bucket.work.wait()
            bucket.flat.mul_(inv)
            for pi, p in enumerate(bucket.params):
                g = bucket.flat[bucket.offsets[pi] : bucket.offsets[pi] + p.numel()].view_as(p)
                if p.grad is None:
                    p.grad = g.clone()
                else:
                    p.grad.copy_(g)

    # ------------------------------------------------------------------ stages 1 / 2
    def _install_flat(self):
        params = self._params()
        unit = _FlatUnit(params, self.rank, self.world_size)
        flat = torch.zeros(unit.padded, dtype=params[0].dtype, device=params[0].device)
        for p, view in zip(params, unit.param_views(flat)):
            view.copy_(p.data)
            p.data = view
        self._flat_params = flat
        self.units = [unit]
        self._hook_gradients(unit)

    # ------------------------------------------------------------------ stage 3
    def _install_stage3(self):
        covered = set()
        modules = []
        for module in self._unit_modules():
            params = [p for p in module.parameters() if id(p) not in self.excluded and id(p) not in covered]
            if params:
                modules.append((module, _FlatUnit(params, self.rank, self.world_size)))
                covered.update(id(p) for p in params)
        self.units = [unit for _, unit in modules]
        rest = [p for p in self._params() if id(p) not in covered]
        root = _FlatUnit(rest, self.rank, self.world_size) if rest else None
        if root is not None:
            self.units.append(root)
        for unit in self.units:
            self._shard(unit)
            self._hook_gradients(unit)
        # Forward order of the module units; the root unit (the LM head and
        # any other leftover) is used after the last one.
        order = [unit for _, unit in modules]
        for k, (module, unit) in enumerate(modules):
            after = order[k + 1] if k + 1 < len(order) else root
            before = order[k - 1] if k > 0 else None
            module.register_forward_pre_hook(lambda _m, _a, u=unit, nxt=after: self._enter(u, nxt))
            module.register_forward_hook(lambda _m, _a, _o, u=unit: self._leave(u))
            module.register_full_backward_pre_hook(lambda _m, _g, u=unit, nxt=before: self._enter(u, nxt))
        if root is not None:
            last = modules[-1][0] if modules else None
            if last is not None:
                last.register_forward_hook(lambda _m, _a, _o, u=root: self._materialize(u))
            else:
                self.model.register_forward_pre_hook(lambda _m, _a, u=root: self._materialize(u))
            self.model.register_forward_hook(lambda _m, _a, _o, u=root: self._leave(u))
            tail = order[-1] if order else None
            self.model.register_full_backward_pre_hook(lambda _m, _g, u=root, nxt=tail: self._enter(u, nxt))

    def _unit_modules(self):
        """Embedding, each block, the final norm (in forward order); a model
        without a ``blocks`` list is one unit."""
        blocks = getattr(self.model, "blocks", None)
        if not isinstance(blocks, torch.nn.ModuleList):
            return [self.model]
        found = [getattr(self.model, "embedding", None), *blocks, getattr(self.model, "norm", None)]
        return [m for m in found if isinstance(m, torch.nn.Module) and _has_parameters(m)]

    @torch.no_grad()
    def _shard(self, unit: _FlatUnit) -> None:
        p0 = unit.params[0]
        unit.local = torch.zeros(unit.chunk, dtype=p0.dtype, device=p0.device)
        for p, (lo, hi, _), view in zip(unit.params, unit.pieces, unit.piece_views(unit.local)):
            if lo < hi:
                view.copy_(p.data.reshape(-1)[lo:hi])
        self._to_local(unit)

    def _to_local(self, unit: _FlatUnit) -> None:
        for p, view in zip(unit.params, unit.piece_views(unit.local)):
            p.data = view
        unit.full = None

    def _start_gather(self, unit: _FlatUnit | None) -> None:
        if unit is None or unit.full is not None or unit.gathering is not None:
            return
        flat = unit.local.new_empty(unit.padded)
        work = dist.all_gather_into_tensor(flat, unit.local, group=self.group, async_op=True)
        unit.gathering = (flat, work)

    @torch.no_grad()
    def _materialize(self, unit: _FlatUnit) -> None:
        if unit.full is not None:
            return
        self._start_gather(unit)
        flat, work = unit.gathering
        work.wait()
        unit.gathering = None
        unit.full = flat
        for p, view in zip(unit.params, unit.param_views(flat)):
            p.data = view

    @torch.no_grad()
    def _enter(self, unit: _FlatUnit, upcoming: _FlatUnit | None) -> None:
        self._materialize(unit)
        if self.prefetch:
            self._start_gather(upcoming)

    @torch.no_grad()
    def _leave(self, unit: _FlatUnit) -> None:
        # The autograd graph holds the parameter objects, not these values;
        # backward's pre-hook materialises them again before they are read.
        if unit.full is not None:
            self._to_local(unit)

    # ------------------------------------------------------------------ gradients (stages 1-3)
    def _hook_gradients(self, unit: _FlatUnit) -> None:
        for p in unit.params:
            p.register_post_accumulate_grad_hook(lambda q, u=unit: self._grad_arrived(u, q))

    @torch.no_grad()
    def _grad_arrived(self, unit: _FlatUnit, p) -> None:
        i = unit.index[id(p)]
        if i in unit.arrived:
            raise RuntimeError(f"a {tuple(p.shape)} parameter received a second gradient in one backward")
        if unit.grad_flat is None:
            unit.grad_flat = unit.new_grad_flat()
        s, n = unit.starts[i], unit.sizes[i]
        unit.grad_flat[s : s + n].copy_(p.grad.reshape(-1))
        p.grad = None
        unit.arrived.add(i)
        if len(unit.arrived) == len(unit.params):
            self._start_reduce(unit)
            if self.stage == 3:
                self._leave(unit)

    def _start_reduce(self, unit: _FlatUnit) -> None:
        self._scale(unit.grad_flat)
        if self.stage == 1:
            unit.scatter = self._all_reduce(unit.grad_flat, async_op=True)
            return
        if unit.grad_chunk is None:
            unit.grad_chunk = unit.grad_flat.new_empty(unit.chunk)
        unit.scatter = dist.reduce_scatter_tensor(unit.grad_chunk, unit.grad_flat, op=dist.ReduceOp.SUM,
                                                  group=self.group, async_op=True)

    def _finish_units(self, total) -> None:
        for unit in self.units:
            if len(unit.arrived) != len(unit.params):
                raise RuntimeError("backward produced no gradient for some parameter of a ZeRO unit")
            if unit.scatter is None:
                self._start_reduce(unit)
        for unit in self.units:
            unit.scatter.wait()
            unit.scatter = None
            unit.reduced = True
            if self.stage == 1:
                unit.grad_flat.div_(total)
                for p, view in zip(unit.params, unit.param_views(unit.grad_flat)):
                    p.grad = view
            else:
                unit.grad_chunk.div_(total)
                for p, view in zip(unit.params, unit.piece_views(unit.grad_chunk)):
                    if view.numel():
                        self.grad_shards[id(p)] = view
            # The next backward fills a fresh buffer (in stage 1 p.grad keeps this one).
            unit.grad_flat = None
