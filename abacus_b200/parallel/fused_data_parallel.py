"""DDP whose gradient all-reduce and AdamW step are NVLink kernels that run
under backward.

Semantics are those of :class:`DataParallel` stage 0 followed by
:class:`AdamW` (``abacus/distributed/data_parallel.py:141-161`` token-weighted
mean gradient, ``abacus/optimizers/adamw.py`` update): after a step every
replica holds the same parameters, equal to one AdamW step on
``sum_r count_r * g_r / sum_r count_r``. The reference all-reduces every
gradient after backward and then steps the optimizer; here the reduction and
the update of each bucket start as soon as backward has produced the bucket's
gradients on every rank.

Layout. All trainable parameters live in one flat fp32 buffer in symmetric
memory (``torch.distributed._symmetric_memory``): every rank maps every peer's
buffer, so a kernel can load and store a peer's memory over NVLink. The
parameters are laid out in reverse registration order (the order in which
backward produces their gradients), each on a 16-byte boundary, and cut into
buckets of about ``bucket_mb`` at parameter boundaries; each bucket's range is
split evenly (in float4 units) between the ranks. Rank r keeps the Adam
moments of its slice of every bucket only (ZeRO-1 sized optimizer state).
Gradients are copied by a post-accumulate hook into a second flat buffer in
the same allocation and the autograd gradient is released at once.

One step, given the learning rate and the token count before backward
(``prepare_step``):

1. When the last gradient of bucket k arrives, an event on the compute stream
   hands the bucket to a communication stream, which runs
   ``symm_barrier`` (every rank has produced bucket k; the first bucket's
   barrier also carries every rank's token count) and ``ar_adamw`` on the
   bucket: rank r reads its slice of every peer's gradient over NVLink, forms
   the token-weighted mean, applies AdamW with its moments and stores the new
   values into every peer's parameter buffer. Buckets launch in index order
   on every rank, so barrier epochs pair up across ranks. The update runs
   while backward computes the earlier layers: once every rank has passed
   bucket k's barrier, no rank's backward reads those parameters again.
2. ``synchronize`` (after backward) launches the buckets that are left
   (zero-filling gradients that backward did not produce), then a final
   ``symm_barrier`` carrying (loss * count, count): every peer's stores into
   this replica have landed and every peer has finished reading this rank's
   gradients before the next forward and backward. The compute stream waits
   for it; the mean loss comes from the exchanged rows, no NCCL call.

``overlap=False`` runs the same kernels, all after backward.

Every device-side wait is bounded (``timeout_ms``); a wait that runs out
sets the device status word, the fused kernels then return without touching
memory, and the next step (or ``check``) raises ``PeerFailure``.
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
# Exchange rows per rank: (loss * count, count) of the final barrier, then
# (count, unused) of the first bucket's barrier, kept apart so that a fast
# rank's next-step count cannot overwrite a row a slow rank is still reading.
_EXCH_COLS = 4


def _round_up(x: int, m: int) -> int:
    return -(-x // m) * m


class _FlatBucket:
    """Flat range [begin, end) of the parameter buffer; rank r owns
    [begin + r * slice, begin + (r + 1) * slice). ``moment_off`` is where this
    rank's slice starts in its moment buffers."""

    def __init__(self, index: int, begin: int, end: int, members: list[int], world: int, rank: int):
        self.index = index
        self.begin, self.end = begin, end
        self.slice = (end - begin) // world
        self.lo = begin + rank * self.slice
        self.hi = self.lo + self.slice
        self.members = members  # parameter indices
        self.arrived: set[int] = set()
        self.launched = False
        self.moment_off = 0


class FusedDataParallel(DataParallel):
    """Stage-0 data parallelism fused with AdamW over NVLink peer memory (CUDA only)."""

    fused_optimizer = True

    def __init__(self, model: torch.nn.Module, dim: str = DIM, token_weighted: bool = True,
                 timeout_ms: float = 60_000.0, bucket_mb: float = 24.0, overlap: bool = True,
                 reduce_ctas: int = 0):
        super().__init__(model, stage=0, dim=dim, token_weighted=token_weighted, bucket_mb=bucket_mb)
        if self.world_size > _MAX_RANKS:
            raise ValueError(f"fused data parallel supports at most {_MAX_RANKS} ranks, got {self.world_size}")
        self.timeout_ms = float(timeout_ms)
        self.overlap = overlap
        # CTAs per bucket reduction while backward runs (0: the kernel's default).
        self.reduce_ctas = int(reduce_ctas)
        self._flat_params: list[torch.nn.Parameter] = []
        self._epoch = 0
        self._status_host = None
        self._status_event = None
        self._stepped = 0
        self._prepared = None  # (lr, betas, eps, wd, step) of the coming backward
        self._next_bucket = 0
        self._pending_optimizer = None

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

        # Backward order: gradients arrive roughly in reverse registration order.
        order = list(reversed(params))
        quantum = _ALIGN * self.world_size
        offsets = {}
        buckets: list[_FlatBucket] = []
        cursor = start = 0
        members: list[int] = []
        for p in order:
            i = len(offsets)
            offsets[id(p)] = cursor
            members.append(i)
            cursor = _round_up(cursor + p.numel(), _ALIGN)
            if (cursor - start) * 4 >= self.bucket_bytes:
                end = _round_up(cursor, quantum)
                buckets.append(_FlatBucket(len(buckets), start, end, members, self.world_size, self.rank))
                cursor = start = end
                members = []
        if members:
            end = _round_up(max(cursor, start + 1), quantum)
            buckets.append(_FlatBucket(len(buckets), start, end, members, self.world_size, self.rank))
            cursor = end
        padded = cursor

        # One symmetric allocation: params | grads | signal slots | exchange rows.
        exch_floats = _round_up(_EXCH_COLS * self.world_size, 64)
        layout = {}
        at = 0
        for name, nbytes in (("param", padded * 4), ("grad", padded * 4), ("signal", _SIGNAL_SLOTS * 4),
                             ("exch", exch_floats * 4)):
            layout[name] = (at, nbytes)
            at = _round_up(at + nbytes, 256)
        raw = symm_mem.empty(at, dtype=torch.uint8, device=device)
        raw.zero_()
        group = self.group if self.group is not None else dist.group.WORLD
        handle = symm_mem.rendezvous(raw, group)
        mine = int(handle.buffer_ptrs[self.rank])
        base = raw.data_ptr() - mine
        if base < 0 or base + at > int(handle.buffer_size):
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
        rows = view("exch", torch.float32)
        self._exch_loss = rows[: 2 * self.world_size].view(self.world_size, 2)
        self._param_ptrs, self._grad_ptrs = peers("param"), peers("grad")
        self._signal_ptrs = peers("signal")
        exch_base = peers("exch")
        self._exch_loss_ptrs = exch_base
        self._exch_count_ptrs = [ptr + 2 * 4 * self.world_size for ptr in exch_base]
        self._exch_counts = rows[2 * self.world_size : 4 * self.world_size].view(self.world_size, 2)

        self._flat_params = order
        self._offsets = [offsets[id(p)] for p in order]
        for p, off in zip(order, self._offsets):
            n = p.numel()
            self._param_flat[off : off + n].copy_(p.data.reshape(-1))
            p.data = self._param_flat[off : off + n].view(p.shape)
        self._index = {id(p): i for i, p in enumerate(order)}
        self._buckets = []  # the stage-0 NCCL buckets are not used
        self.flat_buckets = buckets
        self._bucket_of_param = {}
        for b in buckets:
            for i in b.members:
                self._bucket_of_param[i] = b

        # Moments of the owned slices, bucket after bucket, and per-parameter
        # views of them (the optimizer state: exp_avg of the owned flat range).
        total_slice = 0
        for b in buckets:
            b.moment_off = total_slice
            total_slice += b.slice
        self._exp_avg = torch.zeros(total_slice, dtype=torch.float32, device=device)
        self._exp_avg_sq = torch.zeros(total_slice, dtype=torch.float32, device=device)
        self.owned = {}
        self._moment_views = {}
        for b in buckets:
            for i in b.members:
                p, off = order[i], self._offsets[i]
                begin, stop = max(0, b.lo - off), min(p.numel(), b.hi - off)
                if begin < stop:
                    self.owned[id(p)] = (begin, stop)
                    dest = b.moment_off + off + begin - b.lo
                    self._moment_views[id(p)] = (self._exp_avg[dest : dest + stop - begin],
                                                 self._exp_avg_sq[dest : dest + stop - begin])
        self.grad_shards = None
        for p in order:
            p.register_post_accumulate_grad_hook(self._on_grad_fused)
        self._comm_stream = torch.cuda.Stream(device=device)
        self._status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._status_event = torch.cuda.Event()
        # Every rank's zeroed buffer is in place before any peer writes to it.
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    # ------------------------------------------------------------------ step
    def set_token_count(self, token_count) -> None:
        self._token_count = token_count
        for b in self.flat_buckets:
            b.arrived.clear()
            b.launched = False
        self._next_bucket = 0

    @torch.no_grad()
    def prepare_step(self, optimizer, token_count) -> None:
        """Fix this step's AdamW hyper-parameters and token count before
        backward, so that bucket updates can run under it."""
        self._check_previous()
        self._adopt_state(optimizer)
        step = self._stepped + 1
        for p in self._flat_params:
            st = optimizer.state.get(id(p))
            if st is not None:
                st["step"] += 1
                step = max(step, int(st["step"]))
        self._stepped = step
        self._prepared = (float(optimizer.lr), optimizer.beta1, optimizer.beta2, optimizer.eps,
                          optimizer.weight_decay, step)
        self.set_token_count(token_count)
        device = self._grad_flat.device
        if self.token_weighted:
            count = torch.as_tensor(token_count, device=device).reshape(()).to(torch.float32)
        else:
            count = torch.ones((), device=device, dtype=torch.float32)
        self._count_payload = torch.stack((count, torch.zeros_like(count)))

    @torch.no_grad()
    def _on_grad_fused(self, p):
        i = self._index[id(p)]
        off = self._offsets[i]
        self._grad_flat[off : off + p.numel()].copy_(p.grad.reshape(-1))
        p.grad = None
        bucket = self._bucket_of_param[i]
        bucket.arrived.add(i)
        if self.overlap and self._prepared is not None:
            self._launch_ready()

    def _launch_ready(self) -> None:
        while self._next_bucket < len(self.flat_buckets):
            b = self.flat_buckets[self._next_bucket]
            if len(b.arrived) != len(b.members):
                return
            self._launch_bucket(b)

    def _launch_bucket(self, b: _FlatBucket) -> None:
        compute = torch.cuda.current_stream(self._grad_flat.device)
        self._comm_stream.wait_stream(compute)
        with torch.cuda.stream(self._comm_stream):
            if b.index == 0:
                self._barrier(self._exch_count_ptrs, self._count_payload)
            else:
                self._barrier(None, None)
            lr, beta1, beta2, eps, wd, step = self._prepared
            ext().ar_adamw(
                self._grad_ptrs, self._param_ptrs, self._exch_counts[:, 0], self.token_weighted, self.rank, b.lo, b.hi,
                self._exp_avg[b.moment_off : b.moment_off + b.slice],
                self._exp_avg_sq[b.moment_off : b.moment_off + b.slice], lr, beta1, beta2, eps, wd, step,
                self.reduce_ctas if self.overlap else 0, None,
            )
        b.launched = True
        self._next_bucket += 1

    @torch.no_grad()
    def synchronize(self, loss: torch.Tensor, token_count) -> torch.Tensor:
        """Launch the remaining buckets and the final barrier; returns the global mean loss."""
        if self._prepared is None:
            raise RuntimeError("FusedDataParallel.prepare_step must run before backward")
        if not any(b.arrived for b in self.flat_buckets):
            raise RuntimeError("backward produced no gradients")
        for b in self.flat_buckets[self._next_bucket :]:
            for i in b.members:
                if i not in b.arrived:
                    off = self._offsets[i]
                    self._grad_flat[off : off + self._flat_params[i].numel()].zero_()
                    b.arrived.add(i)
        while self._next_bucket < len(self.flat_buckets):
            self._launch_bucket(self.flat_buckets[self._next_bucket])
        loss32 = loss.detach().reshape(()).to(torch.float32)
        if self.token_weighted:
            count = torch.as_tensor(token_count, device=loss32.device).reshape(()).to(torch.float32)
            payload = torch.stack((loss32 * count, count))
        else:
            payload = torch.stack((loss32, torch.ones_like(loss32)))
        compute = torch.cuda.current_stream(self._grad_flat.device)
        self._comm_stream.wait_stream(compute)
        with torch.cuda.stream(self._comm_stream):
            self._barrier(self._exch_loss_ptrs, payload)
        compute.wait_stream(self._comm_stream)
        payload.record_stream(self._comm_stream)
        self._count_payload.record_stream(self._comm_stream)
        rows = self._exch_loss
        mean = rows[:, 0].sum() / rows[:, 1].sum() if self.token_weighted else rows[:, 0].sum()
        self._prepared = None
        self._status_host.copy_(ext().status_tensor(self._grad_flat.device.index), non_blocking=True)
        self._status_event.record()
        return mean.to(loss.dtype)

    @torch.no_grad()
    def step_optimizer(self, optimizer) -> None:
        """The update already ran per bucket; nothing is left to do."""
        return

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
            self._stepped = max(self._stepped, int(st["step"]))

    def bind_optimizer(self, optimizer) -> None:
        self._adopt_state(optimizer)

    @torch.no_grad()
    def gather_owned(self, pieces: dict[int, torch.Tensor]) -> dict[int, torch.Tensor]:
        """Full flattened tensors from every rank's owned slices (collective)."""
        device = self._grad_flat.device
        chunk = torch.zeros(self._exp_avg.numel(), dtype=torch.float32, device=device)
        for p in self._flat_params:
            views = self._moment_views.get(id(p))
            src = pieces.get(id(p))
            if views is not None and src is not None:
                start = views[0].data_ptr() - self._exp_avg.data_ptr()
                chunk[start // 4 : start // 4 + views[0].numel()].copy_(src.reshape(-1))
        every = chunk.new_empty(chunk.numel() * self.world_size)
        dist.all_gather_into_tensor(every, chunk, group=self.group)
        every = every.view(self.world_size, -1)
        flat = torch.zeros(self._param_flat.numel(), dtype=torch.float32, device=device)
        for b in self.flat_buckets:
            for r in range(self.world_size):
                lo = b.begin + r * b.slice
                flat[lo : lo + b.slice].copy_(every[r, b.moment_off : b.moment_off + b.slice])
        return {id(p): flat[off : off + p.numel()].clone() for p, off in zip(self._flat_params, self._offsets)}

    # ------------------------------------------------------------------ health
    def _barrier(self, exch_ptrs, payload) -> None:
        self._epoch += 1
        if payload is None:
            ext().symm_barrier(self._signal_ptrs, self.rank, 0, self._epoch, self.timeout_ms, [], None)
        else:
            ext().symm_barrier(self._signal_ptrs, self.rank, 0, self._epoch, self.timeout_ms, exch_ptrs,
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
        torch.cuda.synchronize(self._grad_flat.device)
        for p in self._flat_params:
            p.data = p.data.clone()
        self._flat_params = []
        self._raw = self._handle = None
