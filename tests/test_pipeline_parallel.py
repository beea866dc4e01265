"""GPipe over gloo ranks equals the single-process model."""
import pytest
import torch

from _dist import run_ranks
from abacus_b200.distributed.pipeline_parallel import PipelineParallel
from abacus_b200.trainer import Trainer
from abacus_b200.transformer import PipelineStage, Transformer

KW = dict(dim=16, n_heads=2, head_dim=8, n_blocks=4, vocab_size=24, hidden_dim=32)


def _stage_state(single, rank, world):
    """Single-model state re-keyed to a stage's local block indices."""
    per = KW["n_blocks"] // world
    out = {}
    for name, t in single.state_dict().items():
        if name.startswith("blocks."):
            i = int(name.split(".")[1])
            if rank * per <= i < (rank + 1) * per:
                out["blocks." + str(i - rank * per) + name[len(f"blocks.{i}") :]] = t
        elif name.startswith("embedding.") and rank == 0:
            out[name] = t
        elif (name.startswith("norm.") or name == "w_D_vocab") and rank == world - 1:
            out[name] = t
        elif name == "rotary.inv_freq":
            out[name] = t
    return out


def _check(rank, world, micro):
    torch.manual_seed(0)
    single = Transformer(**KW)
    stage = PipelineStage(rank=rank, world_size=world, **KW)
    stage.load_state_dict(_stage_state(single, rank, world))
    tokens = torch.tensor([[3, 5, 7, 1, 2, 9], [6, 0, 11, 2, 23, 4], [1, 1, 2, -100, -100, -100], [7, 8, 9, 10, 11, 12]])
    ts = Trainer(single, total_steps=3)
    tp = Trainer(stage, pipeline=PipelineParallel(stage, n_microbatches=micro), total_steps=3)
    for _ in range(2):
        l1, _ = ts.step(tokens)
        l2, _ = tp.step(tokens)
        if rank == world - 1:
            torch.testing.assert_close(l2, l1, rtol=1e-5, atol=1e-6)
    want = _stage_state(single, rank, world)
    for name, p in stage.named_parameters():
        torch.testing.assert_close(p, want[name], rtol=1e-4, atol=1e-5, msg=name)


@pytest.mark.parametrize("micro", [1, 2, 4])
def test_gpipe_matches_single_process(micro):
    run_ranks(_check, 2, micro)


def test_stage_validation():
    with pytest.raises(ValueError):
        PipelineStage(8, 2, 4, 3, 10, rank=0, world_size=2)
    with pytest.raises(ValueError):
        PipelineStage(8, 2, 4, 4, 10, rank=2, world_size=2)
    s0 = PipelineStage(8, 2, 4, 4, 10, rank=0, world_size=2)
    s1 = PipelineStage(8, 2, 4, 4, 10, rank=1, world_size=2)
    assert hasattr(s0, "embedding") and not hasattr(s0, "w_D_vocab")
    assert hasattr(s1, "w_D_vocab") and not hasattr(s1, "embedding")
    assert [n for n, _ in s1.named_parameters()][0] == "w_D_vocab"
