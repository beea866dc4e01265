"""Checkpoints in the reference's state_dict layout, from sharded layouts."""
import torch

from _dist import run_ranks
from abacus_b200.trainer import Trainer
from abacus_b200.transformer import Transformer
from abacus_b200.utils.checkpoint import full_state_dict, load_checkpoint, save_checkpoint

KW = dict(dim=16, n_heads=4, head_dim=4, n_blocks=2, vocab_size=24, hidden_dim=32)


def test_save_load_resumes_identically(tmp_path):
    torch.manual_seed(0)
    model = Transformer(**KW)
    trainer = Trainer(model, total_steps=6, device="cpu")
    tokens = torch.randint(0, 24, (2, 8))
    trainer.step(tokens)
    path = tmp_path / "ckpt.pt"
    save_checkpoint(path, model, trainer.optimizer, trainer.scheduler)
    l_cont, _ = trainer.step(tokens)
    torch.manual_seed(1)
    fresh = Transformer(**KW)
    t2 = Trainer(fresh, total_steps=6, device="cpu")
    load_checkpoint(path, fresh, t2.optimizer, t2.scheduler)
    l_resumed, _ = t2.step(tokens)
    torch.testing.assert_close(l_resumed, l_cont)
    for a, b in zip(fresh.parameters(), model.parameters()):
        torch.testing.assert_close(a, b)
    saved = torch.load(path, weights_only=False)["model"]
    assert set(saved) == set(model.state_dict())


def _tp_roundtrip(rank, world, path):
    torch.manual_seed(0)
    single = Transformer(**KW)
    torch.manual_seed(0)
    tp = Transformer(**KW, tensor_parallel=True)
    full = full_state_dict(tp)
    for name, t in single.state_dict().items():
        torch.testing.assert_close(full[name], t, msg=name)
    save_checkpoint(path, tp)
    torch.manual_seed(5)
    tp2 = Transformer(**KW, tensor_parallel=True)
    load_checkpoint(path, tp2)
    for (n, a), b in zip(tp2.named_parameters(), tp.parameters()):
        torch.testing.assert_close(a, b, msg=n)


def test_tensor_parallel_checkpoint_is_full_layout(tmp_path):
    run_ranks(_tp_roundtrip, 2, str(tmp_path / "tp.pt"))
    single = Transformer(**KW)
    single.load_state_dict(torch.load(tmp_path / "tp.pt", weights_only=False)["model"])


def _moments(trainer, model):
    return {n: (st["exp_avg"].clone(), st["exp_avg_sq"].clone())
            for n, st in trainer.optimizer.state_dict_by_name(model).items()}


def _tp_optimizer_roundtrip(rank, world, path):
    """Each TP rank's AdamW moments survive a save / load and the runs continue identically."""
    torch.manual_seed(0)
    tp = Transformer(**KW, tensor_parallel=True)
    trainer = Trainer(tp, total_steps=8, device="cpu")
    tokens = torch.randint(0, 24, (2, 8), generator=torch.Generator().manual_seed(3))
    trainer.step(tokens)
    save_checkpoint(path, tp, trainer.optimizer, trainer.scheduler)
    before = _moments(trainer, tp)
    torch.manual_seed(5)
    tp2 = Transformer(**KW, tensor_parallel=True)
    t2 = Trainer(tp2, total_steps=8, device="cpu")
    load_checkpoint(path, tp2, t2.optimizer, t2.scheduler)
    after = _moments(t2, tp2)
    assert set(after) == set(before)
    for name, (m, v) in before.items():
        torch.testing.assert_close(after[name][0], m, msg=name)
        torch.testing.assert_close(after[name][1], v, msg=name)
    l1, _ = trainer.step(tokens)
    l2, _ = t2.step(tokens)
    torch.testing.assert_close(l2, l1)
    for (n, a), b in zip(tp2.named_parameters(), tp.parameters()):
        torch.testing.assert_close(a, b, msg=n)


def test_tensor_parallel_optimizer_state_roundtrip(tmp_path):
    run_ranks(_tp_optimizer_roundtrip, 2, str(tmp_path / "tp_opt.pt"))
    saved = torch.load(tmp_path / "tp_opt.pt", weights_only=False)
    single = Transformer(**KW)
    for name, p in single.named_parameters():
        assert saved["optimizer"][name]["exp_avg"].shape == p.shape, name


def _zero_optimizer_roundtrip(rank, world, path, stage):
    from abacus_b200.distributed.data_parallel import DataParallel

    torch.manual_seed(0)
    model = Transformer(**KW)
    trainer = Trainer(model, DataParallel(model, stage=stage), total_steps=8, device="cpu")
    tokens = torch.randint(0, 24, (2, 8), generator=torch.Generator().manual_seed(10 + rank))
    trainer.step(tokens)
    save_checkpoint(path, model, trainer.optimizer, trainer.scheduler, parallel=trainer.parallel)
    torch.manual_seed(7)
    fresh = Transformer(**KW)
    load_checkpoint(path, fresh)  # weights before the ZeRO wrapper shards them
    t2 = Trainer(fresh, DataParallel(fresh, stage=stage), total_steps=8, device="cpu")
    load_checkpoint(path, fresh, t2.optimizer, t2.scheduler, parallel=t2.parallel)
    for p1, p2 in zip(model.parameters(), fresh.parameters()):
        s1, s2 = trainer.optimizer.state.get(id(p1)), t2.optimizer.state.get(id(p2))
        assert (s1 is None) == (s2 is None)
        if s1 is not None:
            torch.testing.assert_close(s2["exp_avg"].reshape(-1), s1["exp_avg"].reshape(-1))
            torch.testing.assert_close(s2["exp_avg_sq"].reshape(-1), s1["exp_avg_sq"].reshape(-1))
            assert s2["step"] == s1["step"]
    l1, _ = trainer.step(tokens)
    l2, _ = t2.step(tokens)
    torch.testing.assert_close(l2, l1)
    for a, b in zip(t2.parallel.full_parameters(), trainer.parallel.full_parameters()):
        torch.testing.assert_close(a, b)


def test_zero_optimizer_state_roundtrip(tmp_path):
    for stage in (1, 2, 3):
        run_ranks(_zero_optimizer_roundtrip, 2, str(tmp_path / f"zero{stage}.pt"), stage)
    saved = torch.load(tmp_path / "zero2.pt", weights_only=False)
    single = Transformer(**KW)
    for name, p in single.named_parameters():
        assert saved["optimizer"][name]["exp_avg"].shape == p.shape, name
