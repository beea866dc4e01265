"""Data parallelism: DDP (ZeRO-0) and ZeRO-1/2/3, token-weighted.

API and semantics follow ``abacus/distributed/data_parallel.py``: gradients
are the token-weighted mean over every rank's targets (each rank's gradient is
multiplied by its local count, summed, divided by the global count); stage 1
shards the Adam moments, stage 2 also the gradients (reduce-scatter), stage 3
also the parameters, gathered one unit (embedding, each block, final norm,
root leftovers) at a time through module hooks. ``owned`` / ``grad_shards``
feed the ZeRO-aware AdamW exactly as in the reference.

B200-first differences:

* Stage 0 does not concatenate every gradient after backward. Gradients are
  packed into ~25 MB buckets by post-accumulate hooks and each bucket's
  all-reduce is launched asynchronously while backward continues. Buckets are
  launched strictly in index order on every rank, so the NCCL call sequence is
  identical across ranks even when a parameter receives no gradient.
* The loss / token-count reduction is one 2-element all-reduce issued before
  the buckets drain.
* Collectives run on the "dp" group of the installed mesh (the world group
  without one), so DP composes with TP / EP. Parameters listed in
  ``exclude`` (e.g. expert weights sharded over the same ranks) are neither
  broadcast nor reduced.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from abacus_b200.parallel import mesh

DIM = "dp"


def _has_parameters(module: torch.nn.Module) -> bool:
    return next(module.parameters(), None) is not None


class _Partition:
    """A flat parameter range, padded so every rank owns the same number of elements."""

    def __init__(self, params: list[torch.nn.Parameter], rank: int, world_size: int):
        if not params:
            raise ValueError("parameter partition is empty")
        self.params = params
        self.shapes = [tuple(p.shape) for p in params]
        self.numels = [p.numel() for p in params]
        self.offsets = []
        total = 0
        for n in self.numels:
            self.offsets.append(total)
            total += n
        self.total = total
        self.shard = -(-total // world_size)
        self.padded = self.shard * world_size
        lo, hi = rank * self.shard, (rank + 1) * self.shard
        self.owns: list[tuple[int, int]] = []
        self.dests: list[int] = []
        for off, n in zip(self.offsets, self.numels):
            begin, stop = max(0, lo - off), min(n, hi - off)
            if begin >= stop:
                self.owns.append((0, 0))
                self.dests.append(0)
            else:
                self.owns.append((begin, stop))
                self.dests.append(max(off, lo) - lo)
        self.shards: list[torch.Tensor] = []
        self.gathered = False
        self.pending: dict[int, torch.Tensor] = {}
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
    ):
        if not dist.is_initialized():
            raise RuntimeError("Call init_process_group before DataParallel")
        if stage not in (0, 1, 2, 3):
            raise ValueError(f"zero stage must be 0, 1, 2, or 3, got {stage}")
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
        self.partitions: list[_Partition] = []
        self.owned: dict[int, tuple[int, int]] | None = None
        self.grad_shards: dict[int, torch.Tensor] | None = None
        self._token_count = 0
        self._buckets: list[_Bucket] = []
        self._bucket_of: dict[int, tuple[int, int]] = {}
        self._next_launch = 0
        self._hooks_installed = False

    # ------------------------------------------------------------------ helpers
    def _params(self):
        return [p for p in self.model.parameters() if id(p) not in self.excluded]

    def _all_reduce(self, t, async_op=False):
        return dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group, async_op=async_op)

    # ------------------------------------------------------------------ API
    def set_token_count(self, token_count) -> None:
        """This rank's target-token count for the coming backward (int or 0-d tensor)."""
        self._token_count = token_count
        for part in self.partitions:
            part.pending.clear()
            part.reduced = False
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
        self.partitions = []
        if self.stage == 3:
            self._install_stage3()
        else:
            self.partitions.append(_Partition(self._params(), self.rank, self.world_size))
        self.owned = {}
        for part in self.partitions:
            for p, (b, e) in zip(part.params, part.owns):
                if b != e:
                    self.owned[id(p)] = (b, e)
        self.grad_shards = {} if self.stage >= 2 else None

    @torch.no_grad()
    def synchronize(self, loss: torch.Tensor, token_count) -> torch.Tensor:
        """Reduce gradients after backward; returns the global token-weighted mean loss."""
        mean, total = self._mean_loss(loss, token_count)
        if self.stage == 0:
            self._finish_buckets(total)
        elif self.stage == 1:
            self._all_reduce_grads(token_count, total)
        elif self.stage == 2:
            self._reduce_scatter_grads(token_count, total)
        else:
            self._scale_sharded_grads(total)
        return mean

    @torch.no_grad()
    def gather_parameters(self) -> None:
        if self.stage not in (1, 2):
            return
        part = self.partitions[0]
        flat = self._all_gather_unpadded(part, from_shards=False)
        for p, off, n in zip(part.params, part.offsets, part.numels):
            p.data.reshape(-1).copy_(flat[off : off + n])

    @torch.no_grad()
    def full_parameters(self) -> list[torch.Tensor]:
        if self.stage < 3:
            return [p.detach().clone() for p in self.model.parameters()]
        by_id = {}
        for part in self.partitions:
            flat = self._all_gather_unpadded(part, from_shards=True)
            for p, off, n, shape in zip(part.params, part.offsets, part.numels, part.shapes):
                by_id[id(p)] = flat[off : off + n].view(shape).clone()
        return [by_id.get(id(p), p.detach().clone()) for p in self.model.parameters()]

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
            raise RuntimeError("no tokens contributed to the loss")
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

    def _multiplier(self):
        return self._token_count if self.token_weighted else 1.0

    def _launch(self, bucket):
        count = self._multiplier()
        if isinstance(count, torch.Tensor):
            bucket.flat.mul_(count.to(bucket.flat.dtype))
        else:
            bucket.flat.mul_(float(count))
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

    # ------------------------------------------------------------------ stages 1-2
    def _packed_grads(self, part, token_count):
        flat = torch.zeros(part.padded, dtype=part.params[0].dtype, device=part.params[0].device)
        for p, off, n in zip(part.params, part.offsets, part.numels):
            if p.grad is None:
                raise RuntimeError("backward produced no gradient for a parameter")
            flat[off : off + n].copy_(p.grad.reshape(-1))
        flat.mul_(torch.as_tensor(token_count if self.token_weighted else 1.0, dtype=flat.dtype, device=flat.device))
        return flat

    def _all_reduce_grads(self, token_count, total):
        part = self.partitions[0]
        flat = self._packed_grads(part, token_count)
        self._all_reduce(flat)
        flat = flat[: part.total] / total
        for p, off, n in zip(part.params, part.offsets, part.numels):
            p.grad.copy_(flat[off : off + n].view_as(p.grad))

    def _reduce_scatter_grads(self, token_count, total):
        part = self.partitions[0]
        self._scatter_owned_grads(part, self._packed_grads(part, token_count), total)
        for p in part.params:
            p.grad = None

    def _scale_sharded_grads(self, total):
        for part in self.partitions:
            if not part.reduced:
                raise RuntimeError("backward produced no gradient for a parameter")
            part.reduced = False
        for g in self.grad_shards.values():
            g.div_(total)

    def _scatter_owned_grads(self, part, flat, total):
        local = flat.new_empty(part.shard)
        dist.reduce_scatter_tensor(local, flat, op=dist.ReduceOp.SUM, group=self.group)
        if total is not None:
            local.div_(total)
        for p, (b, e), dest in zip(part.params, part.owns, part.dests):
            if b != e:
                self.grad_shards[id(p)] = local[dest : dest + (e - b)].clone()

    # ------------------------------------------------------------------ stage 3
    def _install_stage3(self):
        covered = set()
        for module in self._unit_modules():
            params = [p for p in module.parameters() if id(p) not in self.excluded]
            if not params:
                continue
            part = _Partition(params, self.rank, self.world_size)
            self._materialize(part)
            self.partitions.append(part)
            covered.update(id(p) for p in params)
            self._hook_module(module, part)
        root = [p for p in self._params() if id(p) not in covered]
        if root:
            part = _Partition(root, self.rank, self.world_size)
            self._materialize(part)
            self.partitions.append(part)
            self._hook_root(part)

    def _unit_modules(self):
        blocks = getattr(self.model, "blocks", None)
        if not isinstance(blocks, torch.nn.ModuleList):
            return [self.model]
        modules = []
        emb = getattr(self.model, "embedding", None)
        if emb is not None and _has_parameters(emb):
            modules.append(emb)
        modules.extend(b for b in blocks if _has_parameters(b))
        norm = getattr(self.model, "norm", None)
        if norm is not None and _has_parameters(norm):
            modules.append(norm)
        return modules

    def _materialize(self, part):
        for p, (b, e) in zip(part.params, part.owns):
            shard = p.data.new_empty(0) if b == e else p.data.reshape(-1)[b:e].detach().clone()
            part.shards.append(shard)
        for p, shard in zip(part.params, part.shards):
            p.data = shard
        part.gathered = False

    def _hook_module(self, module, part):
        module.register_forward_pre_hook(lambda _m, _a, part=part: self._gather(part))
        module.register_forward_hook(lambda _m, _a, _o, part=part: self._reshard(part))
        module.register_full_backward_pre_hook(lambda _m, _g, part=part: self._gather(part))
        for p in part.params:
            p.register_post_accumulate_grad_hook(lambda q, part=part: self._on_grad_stage3(q, part))

    def _hook_root(self, part):
        norm = getattr(self.model, "norm", None)
        if isinstance(norm, torch.nn.Module):
            norm.register_forward_hook(lambda _m, _a, _o, part=part: self._gather(part))
        else:
            self.model.register_forward_pre_hook(lambda _m, _a, part=part: self._gather(part))
        self.model.register_forward_hook(lambda _m, _a, _o, part=part: self._reshard(part))
        self.model.register_full_backward_pre_hook(lambda _m, _g, part=part: self._gather(part))
        for p in part.params:
            p.register_post_accumulate_grad_hook(lambda q, part=part: self._on_grad_stage3(q, part))

    @torch.no_grad()
    def _gather(self, part):
        if part.gathered:
            return
        flat = self._all_gather_unpadded(part, from_shards=True)
        for p, off, n, shape in zip(part.params, part.offsets, part.numels, part.shapes):
            p.data = flat[off : off + n].view(shape)
        part.gathered = True

    @torch.no_grad()
    def _reshard(self, part):
        if not part.gathered:
            return
        for p, shard in zip(part.params, part.shards):
            p.data = shard
        part.gathered = False

    @torch.no_grad()
    def _on_grad_stage3(self, p, part):
        if p.grad is None:
            raise RuntimeError("backward produced no gradient for a parameter")
        if id(p) in part.pending:
            raise RuntimeError("gradient accumulated twice for one parameter")
        part.pending[id(p)] = p.grad.detach()
        p.grad = None
        if len(part.pending) != len(part.params):
            return
        flat = torch.zeros(part.padded, dtype=p.dtype, device=p.device)
        for q, off, n in zip(part.params, part.offsets, part.numels):
            flat[off : off + n].copy_(part.pending[id(q)].reshape(-1))
        flat.mul_(torch.as_tensor(self._multiplier(), dtype=flat.dtype, device=flat.device))
        self._scatter_owned_grads(part, flat, None)
        part.pending.clear()
        self._reshard(part)
        part.reduced = True

    def _all_gather_unpadded(self, part, from_shards):
        local = torch.zeros(part.shard, dtype=part.params[0].dtype, device=part.params[0].device)
        for i, (p, (b, e), dest) in enumerate(zip(part.params, part.owns, part.dests)):
            if b == e:
                continue
            src = part.shards[i] if from_shards else p.data.reshape(-1)[b:e]
            local[dest : dest + (e - b)].copy_(src)
        gathered = local.new_empty(part.padded)
        dist.all_gather_into_tensor(gathered, local, group=self.group)
        return gathered[: part.total]
