"""Rank grid with per-dimension process groups, and the hybrid layouts the
reference cannot express (TP x DP, CP x PP, EP over DP ranks), each checked
against a single-process run of the same model."""
import torch

from _dist import run_ranks
from abacus_b200.distributed.data_parallel import DataParallel
from abacus_b200.distributed.pipeline_parallel import PipelineParallel
from abacus_b200.optimizers.adamw import AdamW
from abacus_b200.parallel import mesh
from abacus_b200.trainer import Trainer
from abacus_b200.transformer import PipelineStage, Transformer
from abacus_b200.transformer_moe import TransformerMoe

TP_SLICED = {
    "attention.w_q_DHK": 1, "attention.w_k_DHK": 1, "attention.w_v_DHK": 1, "attention.w_o_HKD": 0,
    "mlp.w_gate_DM": 1, "mlp.w_up_DM": 1, "mlp.w_down_MD": 0,
}


def test_mesh_coordinates_and_groups():
    m = mesh.Mesh(pp=2, dp=2, cp=1, tp=2)
    assert m.size == 8
    for r in range(8):
        assert m.rank_of(m.coords(r)) == r
    assert m.group_ranks("tp", 5) == [4, 5]
    assert m.group_ranks("dp", 5) == [5, 7]
    assert m.group_ranks("pp", 5) == [1, 5]
    m2 = mesh.Mesh(dp=4, ep=2)
    assert m2.group_ranks("ep", 3) == [2, 3]


def _slice(name, full, tp_rank, tp):
    for suffix, axis in TP_SLICED.items():
        if name.endswith(suffix):
            return full.chunk(tp, dim=axis)[tp_rank]
    return full


def _tp_dp(rank, world):
    m = mesh.init_mesh(dp=2, tp=2)
    c = m.coords(rank)
    kw = dict(dim=16, n_heads=4, head_dim=4, n_blocks=2, vocab_size=24, hidden_dim=32)
    batches = [torch.tensor([[1, 5, 7, 2, 9, 4, 3, 8]]), torch.tensor([[6, 0, 11, 2, 23, 4, -100, -100]])]
    torch.manual_seed(0)
    single = Transformer(**kw)
    torch.manual_seed(0)
    model = Transformer(**kw, tensor_parallel=True, sequence_parallel=True)
    trainer = Trainer(model, DataParallel(model, stage=0, bucket_mb=0.01))
    opt = AdamW(single)
    for _ in range(2):
        grads, counts = [], []
        for b in batches:
            scratch = Transformer(**kw)
            scratch.load_state_dict(single.state_dict())
            tgt = torch.cat([b[:, 1:], torch.full_like(b[:, :1], -100)], 1)
            loss = scratch(b.clamp(min=0), targets=tgt)
            loss.backward()
            grads.append([p.grad for p in scratch.parameters()])
            counts.append(int((tgt != -100).sum()))
        for i, p in enumerate(single.parameters()):
            p.grad = sum(g[i] * n for g, n in zip(grads, counts)) / sum(counts)
        opt.step()
        trainer.step(batches[c["dp"]])
    ref = dict(single.named_parameters())
    for name, p in model.named_parameters():
        torch.testing.assert_close(p, _slice(name, ref[name], c["tp"], 2), rtol=1e-4, atol=1e-5, msg=name)


def test_tensor_x_data_parallel():
    run_ranks(_tp_dp, 4)


def _stage_state(state, n_blocks, pp_rank, pp):
    per = n_blocks // pp
    out = {}
    for name, t in state.items():
        if name.startswith("blocks."):
            i = int(name.split(".")[1])
            if pp_rank * per <= i < (pp_rank + 1) * per:
                out["blocks." + str(i - pp_rank * per) + name[len(f"blocks.{i}"):]] = t
        elif name.startswith("embedding.") and pp_rank == 0:
            out[name] = t
        elif (name.startswith("norm.") or name == "w_D_vocab") and pp_rank == pp - 1:
            out[name] = t
        elif name == "rotary.inv_freq":
            out[name] = t
    return out


def _cp_pp(rank, world):
    m = mesh.init_mesh(pp=2, cp=2)
    c = m.coords(rank)
    kw = dict(dim=16, n_heads=2, head_dim=8, n_blocks=2, vocab_size=24, hidden_dim=32)
    torch.manual_seed(0)
    single = Transformer(**kw)
    stage = PipelineStage(rank=c["pp"], world_size=2, context_parallel=True, **kw)
    stage.load_state_dict(_stage_state(single.state_dict(), 2, c["pp"], 2))
    tokens = torch.tensor([[3, 5, 7, 1, 2, 9, 4, 8], [6, 0, 11, 2, 23, 4, 4, -100]])
    ts = Trainer(single, total_steps=3)
    tp = Trainer(stage, pipeline=PipelineParallel(stage, n_microbatches=2), total_steps=3)
    for _ in range(2):
        l1, _ = ts.step(tokens)
        l2, _ = tp.step(tokens)
    want = _stage_state(dict(single.named_parameters()), 2, c["pp"], 2)
    for name, p in stage.named_parameters():
        torch.testing.assert_close(p, want[name], rtol=1e-4, atol=1e-5, msg=name)


def test_context_x_pipeline_parallel():
    run_ranks(_cp_pp, 4)


def _ep_dp(rank, world):
    mesh.init_mesh(dp=2, ep=2)
    kw = dict(dim=8, n_heads=2, head_dim=4, n_blocks=1, vocab_size=16, n_experts=4, top_k=2, hidden_dim=16,
              bias_update_speed=0.0)
    batches = [torch.tensor([[1, 5, 7, 2, 9, 4]]), torch.tensor([[6, 0, 11, 2, 3, -100]])]
    torch.manual_seed(0)
    single = TransformerMoe(**kw)
    torch.manual_seed(0)
    model = TransformerMoe(**kw, expert_parallel=True, expert_data_parallel=True)
    experts = [p for n, p in model.named_parameters() if ".moe.w_" in n]
    dp = DataParallel(model, stage=0, exclude=experts, token_weighted=False)
    trainer = Trainer(model, dp)
    opt = AdamW(single)
    union = torch.cat(batches, 0)
    for _ in range(2):
        single.zero_grad()
        tgt = torch.cat([union[:, 1:], torch.full_like(union[:, :1], -100)], 1)
        single(union.clamp(min=0), targets=tgt).backward()
        opt.step()
        trainer.step(batches[rank])
    ref = dict(single.named_parameters())
    for name, p in model.named_parameters():
        want = ref[name]
        if p.shape != want.shape:
            n = p.shape[0]
            want = want[rank * n : (rank + 1) * n]
        torch.testing.assert_close(p, want, rtol=1e-4, atol=1e-5, msg=name)


def test_expert_parallel_over_data_parallel_ranks():
    run_ranks(_ep_dp, 2)
