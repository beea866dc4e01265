"""Router, MoE and load-balancing semantics (CPU)."""
import math

import pytest
import torch

from abacus_b200.mlp import MLP
from abacus_b200.moe.load_balancing import load_balancing_loss
from abacus_b200.moe.moe import MoE
from abacus_b200.moe.router import Router


def test_bias_steers_selection_and_updates_by_sign():
    router = Router(dim=1, n_experts=4, top_k=2, bias_update_speed=10.0, route_scale=2.5)
    with torch.no_grad():
        router.w_DE.copy_(torch.tensor([[2.0, 0.0, -2.0, 1.0]]))
        router.expert_bias_E.copy_(torch.tensor([0.0, 0.0, 10.0, 0.0]))
    x = torch.ones(1, 4, 1)
    scores = torch.sigmoid(x @ router.w_DE)
    router.train()
    w, idx = router(x)
    assert torch.all(idx[..., 0] == 2) and torch.all(idx[..., 1] == 0)
    chosen = scores.gather(-1, idx)
    torch.testing.assert_close(w, chosen / chosen.sum(-1, keepdim=True) * 2.5)
    # Experts 2 and 0 took all 8 slots: their bias drops by 10, the idle ones rise.
    torch.testing.assert_close(router.expert_bias_E, torch.tensor([-10.0, 10.0, 0.0, 10.0]))
    _, idx2 = router(x)
    assert torch.all(idx2[..., 0] == 3) and torch.all(idx2[..., 1] == 1)


def test_bias_frozen_in_eval_and_with_zero_speed():
    router = Router(4, 3, 1, bias_update_speed=0.0)
    router.train()
    router(torch.randn(2, 3, 4))
    assert torch.all(router.expert_bias_E == 0)
    router = Router(4, 3, 1)
    router.eval()
    router(torch.randn(2, 3, 4))
    assert torch.all(router.expert_bias_E == 0)


def test_single_expert_equals_mlp():
    torch.manual_seed(0)
    moe = MoE(6, n_experts=1, top_k=1, hidden_dim=12)
    mlp = MLP(6, 12)
    with torch.no_grad():
        mlp.w_gate_DM.copy_(moe.w_gate_EDM[0])
        mlp.w_up_DM.copy_(moe.w_up_EDM[0])
        mlp.w_down_MD.copy_(moe.w_down_EMD[0])
    x = torch.randn(2, 5, 6)
    torch.testing.assert_close(moe(x), mlp(x))


def _dense_moe(moe, x):
    """Every expert on every token, combined with the router weights."""
    w, idx = moe.router(x)
    out = torch.zeros_like(x)
    for e in range(moe.n_experts):
        y = (torch.nn.functional.silu(x @ moe.w_gate_EDM[e]) * (x @ moe.w_up_EDM[e])) @ moe.w_down_EMD[e]
        out = out + y * (w * (idx == e)).sum(-1, keepdim=True)
    return out


@pytest.mark.parametrize("router", ["sigmoid", "softmax"])
def test_grouped_moe_matches_dense_combination(router):
    torch.manual_seed(1)
    moe = MoE(8, n_experts=4, top_k=2, hidden_dim=16, bias_update_speed=0.0, router=router)
    moe.eval()
    x = torch.randn(3, 7, 8)
    torch.testing.assert_close(moe(x), _dense_moe(moe, x))


def test_softmax_router_records_aux_loss():
    torch.manual_seed(2)
    router = Router(8, 4, 2, router="softmax", aux_loss_coeff=0.1)
    router.train()
    x = torch.randn(2, 5, 8)
    w, idx = router(x)
    probs = torch.softmax(x @ router.w_DE, -1)
    torch.testing.assert_close(router.aux_loss, load_balancing_loss(probs, idx, 0.1))
    torch.testing.assert_close(w.sum(-1), torch.ones(2, 5))


def test_capacity_factor_drops_overflow_in_token_order():
    torch.manual_seed(3)
    moe = MoE(4, n_experts=2, top_k=1, hidden_dim=8, bias_update_speed=0.0, capacity_factor=0.5)
    with torch.no_grad():
        moe.router.w_DE.zero_()
        moe.router.w_DE[:, 0] = 5.0  # every token prefers expert 0
    x = torch.rand(1, 8, 4) + 0.5
    out = moe(x)
    capacity = math.ceil(0.5 * 8 * 1 / 2)  # 2 tokens
    assert torch.all(out[0, capacity:] == 0)
    assert torch.all(out[0, :capacity] != 0)


def test_load_balancing_loss_values():
    probs = torch.tensor([[0.7, 0.3], [0.2, 0.8], [0.6, 0.4], [0.5, 0.5]])
    idx = torch.tensor([0, 1, 0, 0])
    # f = (3/4, 1/4), p = (0.5, 0.5) -> coeff * E * sum = 0.01 * 2 * 0.5
    torch.testing.assert_close(load_balancing_loss(probs, idx), torch.tensor(0.01))
    assert load_balancing_loss(torch.zeros(0, 3), torch.zeros(0, dtype=torch.long)).item() == 0.0
    with pytest.raises(ValueError):
        load_balancing_loss(probs, torch.zeros(4, 1, 1, dtype=torch.long))


def test_capacity_slabs_match_dynamic_grouping():
    """Static capacity slabs (no host sync) give the dynamic grouping's result
    with the router's capacity mask applied, values and gradients."""
    from abacus_b200.models.moe import _capacity_keep, _grouped_experts, _grouped_experts_capacity

    torch.manual_seed(0)
    t, k, e, d, m = 40, 2, 4, 8, 12
    x = torch.randn(t, d, requires_grad=True)
    idx = torch.randint(0, e, (t, k))
    idx[:, 1] = (idx[:, 0] + 1) % e  # distinct experts per token
    w = torch.rand(t, k, requires_grad=True)
    gate, up, down = (torch.randn(e, d, m) * 0.3).requires_grad_(), (torch.randn(e, d, m) * 0.3).requires_grad_(), \
        (torch.randn(e, m, d) * 0.3).requires_grad_()
    capacity = 15  # < t*k/e = 20 on average: some assignments drop
    keep = _capacity_keep(idx, e, capacity)
    assert not keep.all()
    want = _grouped_experts(x, w * keep, idx, gate, up, down)
    got = _grouped_experts_capacity(x, w * keep, idx, gate, up, down, capacity)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
    gw = torch.autograd.grad(want.square().sum(), (x, w, gate, up, down))
    gg = torch.autograd.grad(got.square().sum(), (x, w, gate, up, down))
    for a, b in zip(gg, gw):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
