"""Fused compute + collective kernels in loopback on ONE GPU.

The tensor-parallel, context-parallel and data-parallel kernels take tables of
peer pointers. Here P emulated ranks live on one GPU: every "peer" buffer is
a separate allocation on cuda:0, and the ranks' kernels are launched one after
another on one stream in dependency order (all pushes before any consumer), so
no kernel ever waits for a kernel that has not already finished: every flag a
consumer waits on is set before it starts. The results are compared with a
PyTorch fp64 / fp32 oracle of the collective followed by the computation
(the multi-GPU tests compare the same kernels across real NVLink peers).

Covered: the sequence-parallel all-gather fused into a waiting GEMM
(``tp_push_rows`` + ``gemm_out_tp`` wait), the GEMM -> reduce-scatter
epilogue with the owner-side reduction (``gemm_out_tp`` scatter +
``tp_reduce_rows``), the context-parallel flash forward over pushed K / V
(``flash_attn_fwd_cp``), the data-parallel reduce + AdamW + broadcast
(``ar_adamw``) and its ZeRO-3 local-slice form, and the expert-parallel
dispatch / grouped experts / combine with static capacity slabs.
"""
import math

import pytest
import torch

from abacus_b200.ops import precision
from abacus_b200.ops._ext import check_status, ext

pytestmark = pytest.mark.gpu

SINGLE = 0
WORLD = 2


def _rel(a, b):
    return ((a.double() - b.double()).abs().max() / b.double().abs().max().clamp(min=1e-30)).item()


def _signals(n=256):
    return [torch.zeros(n, dtype=torch.int32, device="cuda") for _ in range(WORLD)]


def _ptr(t, offset_elems=0):
    return t.data_ptr() + offset_elems * t.element_size()


def _push_all(shards, gathered, sig, off, chunk, seq, epoch):
    """Every emulated rank pushes its shard into every rank's gathered buffer."""
    for r, x in enumerate(shards):
        done = torch.zeros(1, dtype=torch.int32, device="cuda")
        flags = [_ptr(sig[p], off + r) for p in range(WORLD)]
        ext().tp_push_rows(x, [g.data_ptr() for g in gathered], flags, chunk, seq, r, epoch, done)


def _gathered_reference(shards, batch, chunk):
    """(B*L, D): rank r's rows sit at b*L + r*chunk + i."""
    parts = [x.view(batch, chunk, -1) for x in shards]
    return torch.cat(parts, dim=1).reshape(batch * chunk * len(shards), -1)


@pytest.mark.parametrize("passes", [3, 1])
def test_sequence_parallel_gather_into_waiting_gemm(passes):
    torch.manual_seed(0)
    batch, chunk, dim, n = 2, 128, 256, 384
    seq = chunk * WORLD
    shards = [torch.randn(batch * chunk, dim, device="cuda") for _ in range(WORLD)]
    w = torch.randn(dim, n, device="cuda") / math.sqrt(dim)
    gathered = [torch.full((batch * seq, dim), float("nan"), device="cuda") for _ in range(WORLD)]
    sig = _signals()
    off, epoch = 16, 1
    _push_all(shards, gathered, sig, off, chunk, seq, epoch)
    want = _gathered_reference(shards, batch, chunk)
    for r in range(WORLD):
        out = torch.empty(batch * seq, n, device="cuda")
        wait = [_ptr(sig[r], off), 0, epoch, chunk, seq, r]
        ext().gemm_out_tp(out, gathered[r], [w], False, False, SINGLE, 1.0, passes, wait, None)
        torch.cuda.synchronize()
        check_status()
        assert torch.equal(gathered[r], want)
        tol = 1e-5 if passes == 3 else 5e-3
        assert _rel(out, want.double() @ w.double()) < tol


@pytest.mark.parametrize("passes", [3, 1])
def test_gemm_reduce_scatter_epilogue_and_owner_reduction(passes):
    torch.manual_seed(1)
    batch, chunk, k, n = 2, 128, 192, 256
    seq = chunk * WORLD
    rows_local = batch * chunk
    # Row-parallel: every rank holds a partial (B*L, k) input and its own W slice.
    a = [torch.randn(batch * seq, k, device="cuda") for _ in range(WORLD)]
    w = [torch.randn(k, n, device="cuda") / math.sqrt(k) for _ in range(WORLD)]
    residual = [torch.randn(rows_local, n, device="cuda") for _ in range(WORLD)]
    slot = rows_local * n
    staging = [torch.full((WORLD, rows_local, n), float("nan"), device="cuda") for _ in range(WORLD)]
    sig = _signals()
    off = 32
    target = None
    for r in range(WORLD):
        scatter = [chunk, seq]
        scatter += [_ptr(staging[p], r * slot) for p in range(WORLD)]
        scatter += [_ptr(sig[p], off + r) for p in range(WORLD)]
        tiles = ext().gemm_out_tp(staging[r][r], a[r], [w[r]], False, False, SINGLE, 1.0, passes, None, scatter)
        target = int(tiles)
    full = sum(a[r].double() @ w[r].double() for r in range(WORLD)).view(batch, WORLD, chunk, n)
    for p in range(WORLD):
        out = torch.empty(rows_local, n, device="cuda")
        ext().tp_reduce_rows(staging[p], WORLD, sig[p][off : off + WORLD], target, residual[p], out)
        torch.cuda.synchronize()
        check_status()
        want = full[:, p].reshape(rows_local, n) + residual[p].double()
        tol = 1e-5 if passes == 3 else 5e-3
        assert _rel(out, want) < tol


def _attention_reference(q, k, v, q_pos, k_pos, batch, heads, hd):
    qh = q.double().view(batch, -1, heads, hd).transpose(1, 2)
    kh = k.double().view(batch, -1, heads, hd).transpose(1, 2)
    vh = v.double().view(batch, -1, heads, hd).transpose(1, 2)
    s = qh @ kh.transpose(-1, -2) / math.sqrt(hd)
    mask = k_pos.view(1, -1) > q_pos.view(-1, 1)
    s = s.masked_fill(mask, float("-inf"))
    return (torch.softmax(s, dim=-1) @ vh).transpose(1, 2).reshape(q.shape[0], heads * hd)


def _zigzag(rank, world, seq_len):
    chunk = seq_len // (2 * world)
    first = torch.arange(rank * chunk, (rank + 1) * chunk)
    second = torch.arange((2 * world - 1 - rank) * chunk, (2 * world - rank) * chunk)
    return torch.cat((first, second))


def test_context_parallel_flash_forward_over_pushed_kv():
    """Each rank holds a zigzag pair of chunks; K / V of every rank are pushed
    into every rank's gathered buffer and the flash kernel waits for the
    owners' epochs before reading them."""
    precision.set_precision("fp32")
    torch.manual_seed(2)
    batch, heads, hd = 2, 4, 64
    seq_len = 512
    local = seq_len // WORLD  # two chunks of 128 per rank
    hk = heads * hd
    qs, kvs, poss = [], [], []
    for r in range(WORLD):
        pos = _zigzag(r, WORLD, seq_len).cuda()
        poss.append(pos)
        qs.append(torch.randn(batch * local, hk, device="cuda"))
        kvs.append(torch.randn(batch * local, 2 * hk, device="cuda"))
    gathered = [torch.full((batch * seq_len, 2 * hk), float("nan"), device="cuda") for _ in range(WORLD)]
    sig = _signals()
    off, epoch = 64, 1
    _push_all(kvs, gathered, sig, off, local, seq_len, epoch)
    k_pos = torch.cat(poss).to(torch.int64)
    all_kv = _gathered_reference(kvs, batch, local)
    for r in range(WORLD):
        out = torch.empty(batch * local, hk, device="cuda")
        lse = torch.empty(batch, heads, local, device="cuda")
        ext().flash_attn_fwd_cp(qs[r], gathered[r][:, :hk], gathered[r][:, hk:], out, lse, batch, heads, hd, local,
                                seq_len, 1.0 / math.sqrt(hd), poss[r].to(torch.int64), k_pos, 3,
                                [_ptr(sig[r], off), epoch, WORLD, r])
        torch.cuda.synchronize()
        check_status()
        want = _attention_reference(qs[r], all_kv[:, :hk], all_kv[:, hk:], poss[r], k_pos, batch, heads, hd)
        assert _rel(out, want) < 1e-5


def test_data_parallel_reduce_adamw_broadcast():
    """Rank r reduces its slice of both ranks' gradients (token-weighted),
    applies AdamW and stores the result into both replicas."""
    torch.manual_seed(3)
    n = 4096 * 3
    grads = [torch.randn(n, device="cuda") for _ in range(WORLD)]
    w0 = torch.randn(n, device="cuda")
    params = [w0.clone() for _ in range(WORLD)]
    counts = torch.tensor([300.0, 100.0], device="cuda")
    half = n // WORLD
    moments = [(torch.zeros(half, device="cuda"), torch.zeros(half, device="cuda")) for _ in range(WORLD)]
    lr, b1, b2, eps, wd = 1e-3, 0.9, 0.95, 1e-8, 0.1
    for step in (1, 2):
        for r in range(WORLD):
            ext().ar_adamw([g.data_ptr() for g in grads], [p.data_ptr() for p in params], counts, True, r,
                           r * half, (r + 1) * half, moments[r][0], moments[r][1], lr, b1, b2, eps, wd, step, 0, None)
    torch.cuda.synchronize()
    check_status()
    # Oracle: two AdamW steps on the token-weighted mean gradient.
    g = (grads[0].double() * 300 + grads[1].double() * 100) / 400
    w, m, v = w0.double(), torch.zeros_like(g), torch.zeros_like(g)
    for step in (1, 2):
        w = w * (1 - lr * wd)
        m = m + (1 - b1) * (g - m)
        v = b2 * v + (1 - b2) * g * g
        w = w - lr / (1 - b1**step) * m / ((v / (1 - b2**step)).sqrt() + eps)
    assert torch.equal(params[0], params[1])
    assert _rel(params[0], w) < 1e-6


def test_zero3_reduce_scatter_adamw_into_local_slices():
    """ZeRO-3 variant: rank r reduces its slice of both ranks' gradients and
    updates only its own locally stored slice (no replica is written)."""
    torch.manual_seed(4)
    n = 4096 * 2
    half = n // WORLD
    grads = [torch.randn(n, device="cuda") for _ in range(WORLD)]
    w0 = torch.randn(n, device="cuda")
    slices = [w0[r * half : (r + 1) * half].clone() for r in range(WORLD)]
    moments = [(torch.zeros(half, device="cuda"), torch.zeros(half, device="cuda")) for _ in range(WORLD)]
    counts = torch.tensor([100.0, 300.0], device="cuda")
    lr, b1, b2, eps, wd = 2e-3, 0.9, 0.95, 1e-8, 0.1
    dummy = [0] * WORLD
    for r in range(WORLD):
        ext().ar_adamw([g.data_ptr() for g in grads], dummy, counts, True, r, r * half, (r + 1) * half,
                       moments[r][0], moments[r][1], lr, b1, b2, eps, wd, 1, 0, slices[r])
    torch.cuda.synchronize()
    check_status()
    g = (grads[0].double() * 100 + grads[1].double() * 300) / 400
    w = w0.double() * (1 - lr * wd)
    m = (1 - b1) * g
    v = (1 - b2) * g * g
    w = w - lr / (1 - b1) * m / ((v / (1 - b2)).sqrt() + eps)
    assert _rel(torch.cat(slices), w) < 1e-6


def test_expert_parallel_dispatch_grouped_experts_combine():
    """Expert parallelism with static capacity slabs: each emulated rank pushes
    its assignments into the owning rank's expert slabs (ep_push_rows, over
    capacity -> dropped), every rank runs its local experts as grouped
    launches (the up-projection waits for all ranks' pushes, the
    down-projection's epilogue returns rows to their source ranks by row map),
    and each source combines its weighted rows (ep_credit for the dropped ones,
    ep_combine). Oracle: the routed SwiGLU experts in fp64."""
    precision.set_precision("fp32")
    passes = precision.passes()
    torch.manual_seed(5)
    n, dim, hidden, top_k = 96, 128, 256, 2
    local_experts = 2
    n_experts = WORLD * local_experts
    capacity = 40  # below the mean load of 48 per (source, expert): some rows drop
    slab = WORLD * capacity
    rows = local_experts * slab
    xs = [torch.randn(n, dim, device="cuda") for _ in range(WORLD)]
    idx = [torch.stack([torch.randperm(n_experts, device="cuda")[:top_k] for _ in range(n)]) for _ in range(WORLD)]
    wts = [torch.rand(n, top_k, device="cuda") for _ in range(WORLD)]
    wg = [torch.randn(local_experts, dim, hidden, device="cuda") / dim**0.5 for _ in range(WORLD)]
    wu = [torch.randn(local_experts, dim, hidden, device="cuda") / dim**0.5 for _ in range(WORLD)]
    wd = [torch.randn(local_experts, hidden, dim, device="cuda") / hidden**0.5 for _ in range(WORLD)]
    slabs = [torch.zeros(rows, dim, device="cuda") for _ in range(WORLD)]
    metas = [torch.full((rows,), -1, dtype=torch.int32, device="cuda") for _ in range(WORLD)]
    sig = _signals()
    off, epoch = 96, 1
    rets = [torch.zeros(n * top_k, dim, device="cuda") for _ in range(WORLD)]
    counters = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(WORLD)]
    keeps, dropped = [], []
    # Dispatch: every rank pushes before any expert GEMM runs.
    for r in range(WORLD):
        flat_e = idx[r].reshape(-1)
        onehot = torch.nn.functional.one_hot(flat_e, n_experts)
        within = (onehot.cumsum(dim=0) * onehot).sum(dim=-1) - 1
        keep = within < capacity
        dest_rank = torch.where(keep, flat_e // local_experts, -1).to(torch.int32)
        dest_row = ((flat_e % local_experts) * slab + r * capacity + within.clamp(max=capacity - 1)).to(torch.int32)
        done = torch.zeros(1, dtype=torch.int32, device="cuda")
        flags = [_ptr(sig[p], off + r) for p in range(WORLD)]
        ext().ep_push_rows(xs[r], top_k, dest_rank.contiguous(), dest_row.contiguous(), None,
                           [s.data_ptr() for s in slabs], [m.data_ptr() for m in metas], flags, r, epoch, done)
        keeps.append(keep.view(n, top_k))
        dropped.append((~keep).sum().to(torch.int32).reshape(1))
    # Experts: one grouped launch per product on each rank.
    n_tiles = ext().gemm_n_tiles(dim, passes)
    scatter_tail = [r_.data_ptr() for r_ in rets] + [c.data_ptr() for c in counters]
    for p in range(WORLD):
        x3 = slabs[p].view(local_experts, slab, dim)
        g = torch.empty(local_experts, slab, hidden, device="cuda")
        u = torch.empty_like(g)
        h = torch.empty_like(g)
        wait = [_ptr(sig[p], off), 2, epoch, 1, WORLD, p]
        ext().gemm_swiglu_grouped(x3, wg[p], wu[p], g, u, h, passes, wait)
        ext().gemm_grouped(rets[p].view(-1)[:dim].view(1, 1, dim), h, [wd[p]], False, False, SINGLE, 1.0, False, passes,
                           [-1, metas[p].data_ptr()] + scatter_tail)
    # Combine on every source.
    outs = []
    for r in range(WORLD):
        ext().ep_credit(counters[r], dropped[r], n_tiles)
        out = torch.empty(n, dim, device="cuda")
        w_kept = (wts[r] * keeps[r]).contiguous()
        ext().ep_combine(rets[r], w_kept, top_k, counters[r], n * top_k * n_tiles, out)
        outs.append(out)
    torch.cuda.synchronize()
    check_status()
    for r in range(WORLD):
        want = torch.zeros(n, dim, dtype=torch.float64, device="cuda")
        xd = xs[r].double()
        for t in range(n):
            for j in range(top_k):
                if not keeps[r][t, j]:
                    continue
                e = int(idx[r][t, j])
                o, le = divmod(e, local_experts)
                hdn = torch.nn.functional.silu(xd[t] @ wg[o][le].double()) * (xd[t] @ wu[o][le].double())
                want[t] += wts[r][t, j].double() * (hdn @ wd[o][le].double())
        assert _rel(outs[r], want) < 1e-5
    assert sum(int(d) for d in dropped) > 0  # the capacity limit was exercised
