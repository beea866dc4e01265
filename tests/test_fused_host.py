"""Host-side logic of the fused NVLink paths, on CPU: expert-parallel row
placement (every assignment gets a unique row in its expert's slab, ordered by
expert, then source rank, then (token, slot)), receive-buffer headroom, and the
per-step call keys / barrier decisions of the symmetric-memory workspace."""
import torch

from _dist import run_ranks
from abacus_b200.parallel import ep_fused, tp_fused


class _FakeWorkspace:
    def __init__(self, rank, world):
        import torch.distributed as dist

        self.rank, self.world, self.group = rank, world, dist.group.WORLD


def _placement(rank, world):
    import torch.distributed as dist

    n_experts, local, k = 4, 2, 2
    g = torch.Generator().manual_seed(rank + 3)
    indices = torch.randint(0, n_experts, (7 + rank, k), generator=g)
    plan = ep_fused._plan(indices.reshape(-1), n_experts, local, _FakeWorkspace(rank, world))
    flat = indices.reshape(-1)
    # Gather every rank's (expert, dest rank, dest row, source, assignment index).
    rec = torch.stack([flat, plan["dest_rank"].long(), plan["dest_row"].long(),
                       torch.full_like(flat, rank), torch.arange(flat.numel())], dim=1)
    sizes = [torch.zeros(1, dtype=torch.long) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([rec.shape[0]]))
    width = int(max(s.item() for s in sizes))
    padded = torch.full((width, 5), -1, dtype=torch.long)
    padded[: rec.shape[0]] = rec
    out = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(out, padded)
    allrec = torch.cat([o[o[:, 0] >= 0] for o in out])
    for d in range(world):
        mine = allrec[allrec[:, 1] == d]
        rows = mine[:, 2]
        assert sorted(rows.tolist()) == list(range(rows.numel())), "rows of a rank's slabs must tile 0..R-1"
        order = mine[rows.argsort()]
        keys = [(int(e), int(s), int(a)) for e, _, _, s, a in order.tolist()]
        assert keys == sorted(keys), "slab order: expert, then source rank, then (token, slot)"
        assert all(e // local == d for e, _, _ in keys)
    if rank == 0:
        assert plan["recv_max"] <= plan["worst"] and plan["sent_max"] >= 1


def test_ep_row_placement_is_a_permutation_in_slab_order():
    run_ranks(_placement, 2)


def test_receive_capacity_headroom():
    assert ep_fused._capacity(10, 10, 80) == 20  # first use: twice the balanced load
    assert ep_fused._capacity(50, 10, 80) == 80  # skewed: twice the need, capped at the worst case
    assert ep_fused._capacity(15, 10, 80) == 20


class _Ext:
    def __init__(self):
        self.barriers = []

    def symm_barrier(self, ptrs, rank, slot, epoch, timeout, exch, payload):
        self.barriers.append(epoch)


def test_workspace_step_keys_and_barriers(monkeypatch):
    fake = _Ext()
    monkeypatch.setattr(tp_fused, "ext", lambda: fake)
    ws = object.__new__(tp_fused.Workspace)
    ws.rank, ws.world, ws.signal_ptrs = 0, 2, [0, 0]
    ws._calls, ws._backward_seen, ws._barrier_epoch = {}, False, 0
    ws.begin_step()  # first forward: barrier
    assert fake.barriers == [1]
    assert ws.call_key("attn1") == "attn1#0"
    ws.begin_step()  # second microbatch before any backward: fresh keys, no barrier
    assert ws.call_key("attn1") == "attn1#1" and fake.barriers == [1]
    ws._backward_seen = True  # a backward ran: the next forward starts a new step
    ws.begin_step()
    assert fake.barriers == [1, 2] and ws.call_key("attn1") == "attn1#0"
    with torch.no_grad():  # forwards without autograd never wait for a backward
        ws.begin_step()
        assert fake.barriers == [1, 2, 3]
