"""Context parallel (zigzag all-gather KV) equals the single-process model."""
import torch

from _dist import run_ranks
from abacus_b200.distributed.context_parallel import zigzag_positions
from abacus_b200.trainer import Trainer
from abacus_b200.transformer import Transformer


def test_zigzag_positions_balance_chunks():
    assert zigzag_positions(8, 0, 2).tolist() == [0, 1, 6, 7]
    assert zigzag_positions(8, 1, 2).tolist() == [2, 3, 4, 5]
    assert sorted(torch.cat([zigzag_positions(12, r, 3) for r in range(3)]).tolist()) == list(range(12))


def _check(rank, world):
    kw = dict(dim=16, n_heads=2, head_dim=8, n_blocks=2, vocab_size=24, hidden_dim=32)
    torch.manual_seed(0)
    single = Transformer(**kw)
    torch.manual_seed(0)
    cp = Transformer(**kw, context_parallel=True)
    cp.load_state_dict(single.state_dict())
    tokens = torch.tensor([[3, 5, 7, 1, 2, 9, 4, 8], [6, 0, 11, 2, 23, 4, -100, -100]])
    ts, tc = Trainer(single, total_steps=3), Trainer(cp, total_steps=3)
    for _ in range(2):
        l1, _ = ts.step(tokens)
        l2, _ = tc.step(tokens)
        torch.testing.assert_close(l2, l1, rtol=1e-5, atol=1e-6)
    for (n, a), b in zip(cp.named_parameters(), single.parameters()):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5, msg=n)


def test_context_parallel_matches_single_process():
    run_ranks(_check, 2)
