"""Expert parallel with the dispatch fused into the router permutation and the
combine fused into the expert GEMM epilogues (NVLink peer memory), against the
same layer on the NCCL all-to-all path (``abacus/distributed/expert_parallel.py``
semantics): outputs, input / router-weight / expert-weight gradients, and
training steps through the Trainer. Needs two GPUs."""
import os

import pytest
import torch

from _dist import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _layer(device, capacity_factor):
    from abacus_b200.models.moe import MoEExpertParallel

    torch.manual_seed(0)
    return MoEExpertParallel(256, 4, 2, hidden_dim=512, router="softmax", capacity_factor=capacity_factor,
                             data_parallel=True).to(device)


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max().clamp(min=1e-12)).item()


def _check(rank, world):
    from abacus_b200.ops._ext import check_status
    from abacus_b200.parallel import mesh, tp_fused
    from abacus_b200.trainer import Trainer
    from abacus_b200.transformer_moe import TransformerMoe

    device = torch.device("cuda", rank)
    mesh.init_mesh(dp=world, ep=world)
    # capacity 1.25: static capacity slabs (no host sync); None: counts exchange.
    for capacity_factor in (1.25, None):
        fused_layer, plain_layer = _layer(device, capacity_factor), _layer(device, capacity_factor)
        torch.manual_seed(10 + rank)  # each rank routes its own tokens
        x = torch.randn(2, 96, 256, device=device)
        results = []
        for flag, layer in (("1", fused_layer), ("0", plain_layer)):
            os.environ["ABACUS_EP_FUSED"] = flag
            xi = x.clone().requires_grad_()
            for _ in range(3):  # later calls reuse the buffers after a backward
                layer.zero_grad()
                xi.grad = None
                out = layer(xi)
                (out * torch.linspace(-1, 1, out.numel(), device=device).view_as(out)).sum().backward()
            results.append((out.detach(), xi.grad.clone(), [p.grad.clone() for p in layer.parameters()]))
        os.environ["ABACUS_EP_FUSED"] = "1"
        torch.cuda.synchronize()
        check_status()
        (of, xf, gf), (op, xp, gp) = results
        assert _rel(of, op) < 1e-5, capacity_factor
        assert _rel(xf, xp) < 2e-4, capacity_factor
        for (name, _), a, b in zip(fused_layer.named_parameters(), gf, gp):
            assert _rel(a, b) < 2e-4, (name, capacity_factor)
        assert tp_fused._WORKSPACES, "the fused path did not run"

    # Trainer steps of a small EP + DP MoE model on both paths.
    from abacus_b200.distributed.data_parallel import DataParallel

    trainers = []
    for flag in ("1", "0"):
        os.environ["ABACUS_EP_FUSED"] = flag
        torch.manual_seed(0)
        model = TransformerMoe(128, 2, 64, 2, 512, 4, 2, hidden_dim=256, router="softmax", capacity_factor=1.25,
                               expert_parallel=True, expert_data_parallel=True).to(device)
        experts = [p for n, p in model.named_parameters() if ".moe.w_" in n]
        trainers.append(Trainer(model, DataParallel(model, exclude=experts, token_weighted=False), device=device))
    torch.manual_seed(20 + rank)
    for _ in range(2):
        tokens = torch.randint(0, 512, (2, 128), device=device)
        losses = []
        for flag, tr in zip(("1", "0"), trainers):
            os.environ["ABACUS_EP_FUSED"] = flag
            losses.append(tr.step(tokens)[0])
        os.environ["ABACUS_EP_FUSED"] = "1"
        torch.cuda.synchronize()
        check_status()
        torch.testing.assert_close(losses[0], losses[1], rtol=2e-3, atol=1e-4)
    torch.cuda.synchronize()
    tp_fused.reset()


def test_ep_fused_matches_nccl_path():
    run_ranks(_check, 2, timeout_s=60, backend="nccl")
