"""Whole-model checks: the CUDA path (all abacus kernels) against the CPU
oracle path of the same module (plain PyTorch fp32)."""
import copy

import pytest
import torch

from abacus_b200.ops import precision
from abacus_b200.ops._ext import check_status, ext
from abacus_b200.trainer import Trainer
from abacus_b200.transformer import Transformer
from abacus_b200.transformer_moe import TransformerMoe

pytestmark = pytest.mark.gpu


def _err(a, b):
    return ((a.double() - b.double()).abs().max() / b.double().abs().max().clamp(min=1e-30)).item()


def _loss_and_grads(model, tokens):
    model.zero_grad()
    targets = torch.cat([tokens[:, 1:], torch.full_like(tokens[:, :1], -100)], 1)
    loss = model(tokens.clamp(min=0), targets=targets)
    loss.backward()
    return loss.detach().cpu(), {n: p.grad.detach().cpu() for n, p in model.named_parameters()}


@pytest.mark.parametrize("mode,tol", [("fp32", 2e-4), ("tf32", 3e-2)])
def test_dense_model_cuda_matches_cpu_oracle(mode, tol):
    torch.manual_seed(0)
    cpu = Transformer(dim=256, n_heads=4, head_dim=64, n_blocks=2, vocab_size=1024, hidden_dim=512, init_std=0.02)
    gpu = copy.deepcopy(cpu).cuda()
    tokens = torch.randint(0, 1024, (2, 192))
    tokens[1, 150:] = -100
    precision.set_precision(mode)
    try:
        before = ext().launch_count()
        lg, gg = _loss_and_grads(gpu, tokens.cuda())
        launched = ext().launch_count() - before
    finally:
        precision.set_precision("fp32")
    torch.cuda.synchronize()
    check_status()
    lc, gc = _loss_and_grads(cpu, tokens)
    assert launched > 20  # every op ran on the abacus kernels
    assert abs(lg.item() - lc.item()) / abs(lc.item()) < tol
    for name, g in gc.items():
        assert _err(gg[name], g) < 10 * tol, name


def test_trainer_steps_cuda_match_cpu():
    torch.manual_seed(1)
    kw = dict(dim=128, n_heads=2, head_dim=64, n_blocks=2, vocab_size=512, hidden_dim=256)
    cpu = Transformer(**kw)
    gpu = copy.deepcopy(cpu)
    tc, tg = Trainer(cpu, total_steps=5, device="cpu"), Trainer(gpu, total_steps=5)
    tokens = torch.randint(0, 512, (4, 128))
    for _ in range(3):
        lc, _ = tc.step(tokens)
        lg, _ = tg.step(tokens)
        assert abs(lg.item() - lc.item()) < 1e-3 * abs(lc.item())
    for (n, a), b in zip(gpu.named_parameters(), cpu.parameters()):
        assert _err(a.detach().cpu(), b.detach()) < 1e-3, n


def test_moe_model_runs_on_cuda():
    torch.manual_seed(2)
    cpu = TransformerMoe(dim=128, n_heads=2, head_dim=64, n_blocks=1, vocab_size=256, n_experts=4, top_k=2,
                         hidden_dim=256, router="softmax", capacity_factor=1.25)
    gpu = copy.deepcopy(cpu).cuda()
    tokens = torch.randint(0, 256, (2, 128))
    lg, gg = _loss_and_grads(gpu, tokens.cuda())
    lc, gc = _loss_and_grads(cpu, tokens)
    assert abs(lg.item() - lc.item()) < 1e-3 * abs(lc.item())
    for name, g in gc.items():
        assert _err(gg[name], g) < 5e-3, name
