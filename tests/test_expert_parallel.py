"""Expert parallelism on 4 gloo ranks equals the single-process MoE: outputs,
input gradients and parameter gradients (expert grads compared per shard)."""
import pytest
import torch

from _dist import run_ranks
from abacus_b200.moe.moe import MoE, MoEExpertParallel
from abacus_b200.transformer_moe import TransformerMoe


def _compare(reference, parallel, rank):
    ref = dict(reference.named_parameters())
    for name, p in parallel.named_parameters():
        rp = ref[name]
        if p.shape == rp.shape:
            torch.testing.assert_close(p, rp)
            if rp.grad is not None or p.grad is not None:
                torch.testing.assert_close(p.grad, rp.grad, msg=name)
        else:
            n = p.shape[0]
            torch.testing.assert_close(p, rp[rank * n : (rank + 1) * n])
            if rp.grad is not None:
                torch.testing.assert_close(p.grad, rp.grad[rank * n : (rank + 1) * n], msg=name)


def _pair(reference, parallel, x, rank):
    reference.train()
    parallel.train()
    xr = x.clone().requires_grad_(True)
    xp = x.clone().requires_grad_(True)
    for _ in range(2):
        yr, yp = reference(xr), parallel(xp)
        yr.sum().backward()
        yp.sum().backward()
        torch.testing.assert_close(yp, yr)
        torch.testing.assert_close(xp.grad, xr.grad)
        _compare(reference, parallel, rank)
        reference.zero_grad()
        parallel.zero_grad()
        xr.grad = xp.grad = None


def _check(rank, world):
    with pytest.raises(ValueError, match="1 expert on each rank"):
        MoEExpertParallel(dim=4, n_experts=world + 1, top_k=1)
    cases = [
        dict(top_k=1, bias_update_speed=0.25),
        dict(top_k=2, bias_update_speed=0.25, route_scale=1.5),
        dict(top_k=2, router="softmax", capacity_factor=1.25),
    ]
    for seed, kw in enumerate(cases):
        torch.manual_seed(seed)
        reference = MoE(dim=4, n_experts=world, hidden_dim=8, **kw)
        torch.manual_seed(seed)
        parallel = MoEExpertParallel(dim=4, n_experts=world, hidden_dim=8, **kw)
        _pair(reference, parallel, torch.randn(2, 3, 4), rank)  # 6 tokens over 4 ranks: 2, 2, 1, 1
        _pair(reference, parallel, torch.randn(1, 1, 4), rank)  # 3 empty shards
    torch.manual_seed(9)
    reference = MoE(dim=4, n_experts=world, top_k=1, hidden_dim=8, bias_update_speed=0.0)
    torch.manual_seed(9)
    parallel = MoEExpertParallel(dim=4, n_experts=world, top_k=1, hidden_dim=8, bias_update_speed=0.0)
    with torch.no_grad():  # every token to expert 0
        reference.router.w_DE.fill_(-8)
        reference.router.w_DE[:, 0] = 8
        parallel.router.w_DE.copy_(reference.router.w_DE)
    _pair(reference, parallel, torch.randn(2, 3, 4), rank)
    kw = dict(dim=8, n_heads=2, head_dim=4, n_blocks=1, vocab_size=16, n_experts=world, top_k=1, bias_update_speed=0.25)
    torch.manual_seed(3)
    ref_model = TransformerMoe(**kw)
    torch.manual_seed(3)
    par_model = TransformerMoe(**kw, expert_parallel=True)
    tokens = torch.randint(0, 16, (2, 5))
    ref_model.train()
    par_model.train()
    for _ in range(2):
        lr_, lp = ref_model(tokens), par_model(tokens)
        lr_.sum().backward()
        lp.sum().backward()
        torch.testing.assert_close(lp, lr_)
        _compare(ref_model, par_model, rank)
        ref_model.zero_grad()
        par_model.zero_grad()


def test_expert_parallel_matches_single_process():
    run_ranks(_check, 4)


def test_one_process_expert_parallel_falls_back_to_moe():
    torch.manual_seed(0)
    reference = MoE(dim=4, n_experts=4, top_k=2, hidden_dim=8, bias_update_speed=0.1)
    torch.manual_seed(0)
    parallel = MoEExpertParallel(dim=4, n_experts=4, top_k=2, hidden_dim=8, bias_update_speed=0.1)
    reference.train()
    parallel.train()
    x = torch.randn(2, 3, 4)
    torch.testing.assert_close(parallel(x), reference(x))
    torch.testing.assert_close(parallel.router.expert_bias_E, reference.router.expert_bias_E)
