"""Checkpoint interoperability with the reference framework itself.

The reference is imported from ``baseline/_ref`` (an unmodified copy of its
``abacus`` package); the tests skip when it is absent. Models are built from
seed 0 on both sides; a ``state_dict`` written by either framework must load
strictly into the other and give the same logits (CPU, fp32). The sharded
layouts (tensor-parallel heads / MLP hidden, expert-parallel experts) are
gathered by ``abacus_b200.utils.checkpoint`` into the reference's single-rank
layout and must load into the reference's unsharded model.
"""
import os
import sys

import pytest
import torch

from _dist import run_ranks

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "abacus")),
                                reason="reference not installed in baseline/_ref")

DENSE = dict(dim=32, n_heads=4, head_dim=8, n_blocks=2, vocab_size=64)
MOE = dict(dim=32, n_heads=4, head_dim=8, n_blocks=2, vocab_size=64, n_experts=2, top_k=1, hidden_dim=48)


def _reference():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import abacus.transformer as rt
    import abacus.transformer_moe as rtm

    return rt, rtm


def _tokens():
    return torch.randint(0, 64, (2, 12), generator=torch.Generator().manual_seed(1))


def _close(a, b):
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)


def test_dense_state_dict_loads_both_ways():
    from abacus_b200.transformer import Transformer

    rt, _ = _reference()
    torch.manual_seed(0)
    ref = rt.Transformer(**DENSE).eval()
    torch.manual_seed(0)
    ours = Transformer(**DENSE).eval()
    assert set(ref.state_dict()) == set(ours.state_dict())
    for name, t in ref.state_dict().items():
        assert ours.state_dict()[name].shape == t.shape, name
    # reference -> abacus_b200
    ours.load_state_dict(ref.state_dict(), strict=True)
    with torch.no_grad():
        _close(ours(_tokens()), ref(_tokens()))
    # abacus_b200 -> reference (after perturbing ours, so the copy is visible)
    with torch.no_grad():
        for p in ours.parameters():
            p.add_(0.01 * torch.randn_like(p))
    ref.load_state_dict(ours.state_dict(), strict=True)
    with torch.no_grad():
        _close(ref(_tokens()), ours(_tokens()))


def test_moe_state_dict_loads_both_ways():
    from abacus_b200.transformer_moe import TransformerMoe

    _, rtm = _reference()
    torch.manual_seed(0)
    ref = rtm.TransformerMoe(**MOE).eval()
    torch.manual_seed(0)
    ours = TransformerMoe(**MOE).eval()
    assert set(ref.state_dict()) == set(ours.state_dict())
    ours.load_state_dict(ref.state_dict(), strict=True)
    with torch.no_grad():
        _close(ours(_tokens()), ref(_tokens()))
    ref.load_state_dict(ours.state_dict(), strict=True)
    with torch.no_grad():
        _close(ref(_tokens()), ours(_tokens()))


def _tensor_parallel_interop(rank, world, path):
    from abacus_b200.transformer import Transformer
    from abacus_b200.utils.checkpoint import full_state_dict, load_checkpoint

    rt, _ = _reference()
    torch.manual_seed(0)
    ref = rt.Transformer(**DENSE).eval()
    # Gathered TP shards load into the reference's unsharded model, which
    # then matches the single-rank model of the same seed (TP slices the full
    # initialisation).
    torch.manual_seed(3)
    tp = Transformer(**DENSE, tensor_parallel=True).eval()
    torch.manual_seed(3)
    single = Transformer(**DENSE).eval()
    probe = rt.Transformer(**DENSE).eval()
    probe.load_state_dict(full_state_dict(tp), strict=True)
    with torch.no_grad():
        _close(probe(_tokens()), single(_tokens()))
    # A reference checkpoint loads into the sharded model and gives the
    # reference's logits.
    if rank == 0:
        torch.save({"model": ref.state_dict()}, path)
    torch.distributed.barrier()
    load_checkpoint(path, tp)
    with torch.no_grad():
        _close(tp(_tokens()), ref(_tokens()))


def test_tensor_parallel_layout_interoperates(tmp_path):
    run_ranks(_tensor_parallel_interop, 2, str(tmp_path / "ref_dense.pt"))


def _expert_parallel_interop(rank, world, path):
    from abacus_b200.transformer_moe import TransformerMoe
    from abacus_b200.utils.checkpoint import full_state_dict, load_checkpoint

    _, rtm = _reference()
    torch.manual_seed(0)
    ref = rtm.TransformerMoe(**MOE).eval()
    if rank == 0:
        torch.save({"model": ref.state_dict()}, path)
    torch.distributed.barrier()
    torch.manual_seed(4)
    ep = TransformerMoe(**MOE, expert_parallel=True).eval()
    load_checkpoint(path, ep)
    with torch.no_grad():
        _close(ep(_tokens()), ref(_tokens()))
    # And the gathered expert shards load strictly into the reference.
    probe = rtm.TransformerMoe(**MOE).eval()
    probe.load_state_dict(full_state_dict(ep), strict=True)
    with torch.no_grad():
        _close(probe(_tokens()), ref(_tokens()))


def test_expert_parallel_layout_interoperates(tmp_path):
    run_ranks(_expert_parallel_interop, 2, str(tmp_path / "ref_moe.pt"))
