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
