"""Tensor parallel (with and without sequence parallel) on gloo ranks equals the
single-process model: loss, sliced gradients and parameters after a step."""
import pytest
import torch

from _dist import run_ranks
from abacus_b200.distributed.tensor_parallel import _AllReduceGrads, _SumOutputs
from abacus_b200.trainer import Trainer
from abacus_b200.transformer import Transformer

TP_SLICED = {
    "attention.w_q_DHK": 1, "attention.w_k_DHK": 1, "attention.w_v_DHK": 1, "attention.w_o_HKD": 0,
    "mlp.w_gate_DM": 1, "mlp.w_up_DM": 1, "mlp.w_down_MD": 0,
}


def _slice(name, full, rank, world):
    for suffix, axis in TP_SLICED.items():
        if name.endswith(suffix):
            return full.chunk(world, dim=axis)[rank]
    return full


def _check(rank, world, sp):
    kw = dict(dim=16, n_heads=4, head_dim=4, n_blocks=2, vocab_size=24, hidden_dim=32)
    torch.manual_seed(0)
    single = Transformer(**kw)
    torch.manual_seed(0)
    parallel = Transformer(**kw, tensor_parallel=True, sequence_parallel=sp)
    for name, p in parallel.named_parameters():
        torch.testing.assert_close(p, _slice(name, dict(single.named_parameters())[name], rank, world))
    tokens = torch.tensor([[3, 5, 7, 1, 2, 9, 4, 8], [6, 0, 11, 2, 23, 4, 4, 1]])
    t_single, t_par = Trainer(single, total_steps=4), Trainer(parallel, total_steps=4)
    for _ in range(2):
        l1, _ = t_single.step(tokens)
        l2, _ = t_par.step(tokens)
        torch.testing.assert_close(l2, l1, rtol=1e-5, atol=1e-6)
    singles = dict(single.named_parameters())
    for name, p in parallel.named_parameters():
        torch.testing.assert_close(p, _slice(name, singles[name], rank, world), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("sp", [False, True])
def test_tensor_parallel_matches_single_process(sp):
    run_ranks(_check, 2, sp)


def _gradcheck(rank, world):
    x = torch.randn(2, 3, 4, dtype=torch.double, requires_grad=True)
    assert torch.autograd.gradcheck(_SumOutputs.apply, (x,))
    assert torch.autograd.gradcheck(_AllReduceGrads.apply, (x,))


def test_tp_autograd_functions_gradcheck_single_rank():
    run_ranks(_gradcheck, 1)
