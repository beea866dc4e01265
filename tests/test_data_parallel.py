"""DDP and ZeRO-1/2/3 on 2 gloo ranks: every stage must equal one AdamW step
on the token-weighted mean gradient of both ranks' batches."""
import torch
import torch.distributed as dist

from _dist import run_ranks
from abacus_b200.distributed.data_parallel import DataParallel
from abacus_b200.optimizers.adamw import AdamW
from abacus_b200.trainer import Trainer
from abacus_b200.transformer import Transformer

BATCHES = [
    torch.tensor([[1, 2, 3, 4, 5, 6, 7], [8, 9, 10, 11, 12, 13, 14]]),
    torch.tensor([[1, 2, 3, 4, -100, -100, -100], [9, 3, -100, -100, -100, -100, -100]]),
]


def _make():
    return Transformer(dim=16, n_heads=2, head_dim=8, n_blocks=2, vocab_size=20, hidden_dim=24)


def _grads(model, tokens):
    model.zero_grad()
    logits = model(tokens.clamp(min=0))
    targets = tokens[:, 1:]
    loss = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), targets.reshape(-1))
    loss.backward()
    return loss.detach(), int((targets != -100).sum()), [p.grad.clone() for p in model.parameters()]


def _check(rank, world, stage):
    torch.manual_seed(0)
    model = _make()
    reference = _make()
    reference.load_state_dict(model.state_dict())
    ref_opt = AdamW(reference)
    trainer = Trainer(model, DataParallel(model, stage=stage, bucket_mb=0.01))
    for _ in range(2):
        scratch = _make()
        per_rank = []
        for b in BATCHES:
            scratch.load_state_dict(reference.state_dict())
            per_rank.append(_grads(scratch, b))
        total = sum(c for _, c, _ in per_rank)
        for i, p in enumerate(reference.parameters()):
            p.grad = sum(g[i] * c for _, c, g in per_rank) / total
        ref_opt.step()
        loss, _ = trainer.step(BATCHES[rank])
        torch.testing.assert_close(loss, sum(l * c for l, c, _ in per_rank) / total)
        for got, want in zip(trainer.parallel.full_parameters(), reference.parameters()):
            torch.testing.assert_close(got, want, rtol=2e-5, atol=2e-6)


def _all_stages(rank, world):
    for stage in (0, 1, 2, 3):
        _check(rank, world, stage)


def test_zero_stages_equal_token_weighted_adamw():
    run_ranks(_all_stages, 2)


def _dp_owned(rank, world):
    torch.manual_seed(0)
    model = _make()
    dp = DataParallel(model, stage=2)
    dp.broadcast_parameters()
    total = sum(p.numel() for p in model.parameters())
    owned = sum(e - b for b, e in dp.owned.values())
    counts = [torch.zeros(1, dtype=torch.long) for _ in range(world)]
    dist.all_gather(counts, torch.tensor([owned]))
    assert sum(int(c) for c in counts) == total


def test_owned_slices_partition_every_parameter():
    run_ranks(_dp_owned, 2)


def _fused_needs_cuda(rank, world):
    import pytest

    from abacus_b200.distributed.data_parallel import FusedDataParallel

    with pytest.raises(RuntimeError, match="CUDA"):
        model = _make()
        Trainer(model, FusedDataParallel(model), device="cpu")


def test_fused_data_parallel_rejects_cpu_parameters():
    run_ranks(_fused_needs_cuda, 2)
