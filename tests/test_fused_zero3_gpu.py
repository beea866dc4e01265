"""Fused ZeRO-3 (push all-gather per unit, reduce-scatter fused with the
partitioned AdamW under backward, NVLink peer memory) against the reference
semantics: one AdamW step on the token-weighted mean gradient of every rank's
batch (``abacus/distributed/data_parallel.py`` stage 3). The 1-rank case runs
on one GPU; the 2-rank case needs two GPUs (NCCL, rank r on cuda:r, every peer
wait bounded)."""
import pytest
import torch

from _dist import run_ranks

BATCHES = [
    torch.tensor([[1, 2, 3, 4, 5, 6, 7, 8] * 8, [9, 10, 11, 12, 13, 14, 15, 16] * 8]),
    torch.tensor([[1, 2, 3, 4] * 8 + [-100] * 32, [9, 3] * 4 + [-100] * 56]),
]


def _make(device):
    from abacus_b200.transformer import Transformer

    torch.manual_seed(0)
    return Transformer(dim=128, n_heads=2, head_dim=64, n_blocks=2, vocab_size=512, hidden_dim=256).to(device)


def _reference_step(reference, opt, batches, device):
    from abacus_b200.trainer import shifted_targets

    per_rank = []
    snapshot = {k: v.clone() for k, v in reference.state_dict().items()}
    for b in batches:
        reference.load_state_dict(snapshot)
        reference.zero_grad()
        tokens = b.to(device)
        targets = shifted_targets(tokens)
        count = (targets != -100).sum()
        loss = reference(tokens.clamp(min=0), targets=targets, normalizer=count.to(torch.float32))
        loss.backward()
        per_rank.append((loss.detach(), int(count), [p.grad.clone() for p in reference.parameters()]))
    reference.load_state_dict(snapshot)
    total = sum(c for _, c, _ in per_rank)
    for i, p in enumerate(reference.parameters()):
        p.grad = sum(g[i] * c for _, c, g in per_rank) / total
    opt.step()
    return sum(l * c for l, c, _ in per_rank) / total


def _check(rank, world):
    from abacus_b200.distributed.data_parallel import FusedZero3
    from abacus_b200.ops._ext import check_status
    from abacus_b200.optimizers.adamw import AdamW
    from abacus_b200.trainer import Trainer

    device = torch.device("cuda", rank)
    model = _make(device)
    reference = _make(device)
    ref_opt = AdamW(reference)
    parallel = FusedZero3(model, timeout_ms=20_000)
    trainer = Trainer(model, parallel, device=device)
    batches = BATCHES[:world]
    for _ in range(3):
        want_loss = _reference_step(reference, ref_opt, batches, device)
        loss, _ = trainer.step(batches[rank])
        torch.testing.assert_close(loss, want_loss, rtol=1e-5, atol=1e-6)
        for got, want in zip(parallel.full_parameters(), reference.parameters()):
            torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
    parallel.check()
    torch.cuda.synchronize()
    check_status()
    parallel.release()


@pytest.mark.gpu
def test_fused_zero3_one_rank_matches_adamw():
    run_ranks(_check, 1, timeout_s=60, backend="nccl")


@pytest.mark.gpu
@pytest.mark.multigpu
def test_fused_zero3_two_ranks_match_token_weighted_adamw():
    run_ranks(_check, 2, timeout_s=90, backend="nccl")
