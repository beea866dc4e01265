"""Context parallel with the K/V gather fused into the flash kernel's loads
and the dK/dV reduce-scatter fused into its backward stores, against the same
model on the NCCL all-gather path (``abacus/distributed/context_parallel.py``
semantics). Two microbatches run forward before one backward, as in a
pipeline step, so each call must keep its own buffers. Needs two GPUs."""
import os

import pytest
import torch

from _dist import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _model(device):
    from abacus_b200.transformer import Transformer

    torch.manual_seed(0)
    return Transformer(dim=256, n_heads=4, head_dim=64, n_blocks=2, vocab_size=512, context_parallel=True,
                       hidden_dim=512).to(device)


def _check(rank, world):
    from abacus_b200.ops._ext import check_status
    from abacus_b200.parallel import mesh, tp_fused
    from abacus_b200.parallel.pipeline_parallel import context_parallel_targets
    from abacus_b200.trainer import Trainer

    device = torch.device("cuda", rank)
    mesh.init_mesh(cp=world)
    fused_model, plain_model = _model(device), _model(device)
    torch.manual_seed(1)
    micro = [torch.randint(0, 512, (1, 512), device=device) for _ in range(2)]
    micro[1][0, 400:] = -100
    results = []
    for flag, model in (("1", fused_model), ("0", plain_model)):
        os.environ["ABACUS_CP_FUSED"] = flag
        model.zero_grad()
        total = torch.zeros((), device=device)
        for tokens in micro:  # two forwards, then one backward
            targets = context_parallel_targets(tokens, rank, world)
            count = torch.tensor(float(sum(int((context_parallel_targets(t, r, world) != -100).sum())
                                           for t in [tokens] for r in range(world))), device=device)
            total = total + model(tokens.clamp(min=0), targets=targets, normalizer=count)
        total.backward()
        results.append(total.detach())
    os.environ["ABACUS_CP_FUSED"] = "1"
    torch.cuda.synchronize()
    check_status()
    torch.testing.assert_close(results[0], results[1], rtol=1e-5, atol=1e-6)
    for (name, a), b in zip(fused_model.named_parameters(), plain_model.parameters()):
        scale = b.grad.abs().max().clamp(min=1e-12)
        err = ((a.grad - b.grad).abs().max() / scale).item()
        assert err < 2e-4, (name, err)
    assert tp_fused._WORKSPACES, "the fused path did not run"
    # Full steps through the public Trainer (CP branch) on the fused path.
    fused, plain = Trainer(fused_model, None, device=device), Trainer(plain_model, None, device=device)
    for tokens in micro:
        os.environ["ABACUS_CP_FUSED"] = "1"
        loss_f, _ = fused.step(tokens)
        os.environ["ABACUS_CP_FUSED"] = "0"
        loss_p, _ = plain.step(tokens)
        os.environ["ABACUS_CP_FUSED"] = "1"
        torch.cuda.synchronize()
        check_status()
        torch.testing.assert_close(loss_f, loss_p, rtol=2e-3, atol=1e-4)
    torch.cuda.synchronize()
    tp_fused.reset()


def test_cp_fused_matches_nccl_path():
    run_ranks(_check, 2, timeout_s=60, backend="nccl")
