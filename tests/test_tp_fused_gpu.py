"""Tensor + sequence parallel with the collectives fused into the GEMMs over
NVLink peer memory, against the same TP+SP model on the NCCL collectives
(``abacus/distributed/tensor_parallel.py`` semantics): losses and gradients
must agree (gradients, not post-AdamW parameters: AdamW's first step maps any
last-bit difference of a near-zero gradient to a full +-lr update), and
training steps through the Trainer must keep agreeing in loss. Needs two GPUs."""
import os

import pytest
import torch

from _dist import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _model(device):
    from abacus_b200.transformer import Transformer

    torch.manual_seed(0)
    return Transformer(dim=256, n_heads=4, head_dim=64, n_blocks=2, vocab_size=512, tensor_parallel=True,
                       sequence_parallel=True, hidden_dim=512).to(device)


def _check(rank, world):
    from abacus_b200.ops._ext import check_status
    from abacus_b200.parallel import mesh, tp_fused
    from abacus_b200.trainer import Trainer

    from abacus_b200.trainer import shifted_targets

    device = torch.device("cuda", rank)
    mesh.init_mesh(tp=world)
    fused_model, plain_model = _model(device), _model(device)
    torch.manual_seed(1)
    batches = [torch.randint(0, 512, (2, 256)) for _ in range(3)]
    batches[1][1, 200:] = -100  # padding: fewer targets on one row
    for tokens in batches[:2]:
        tokens = tokens.to(device)
        targets = shifted_targets(tokens)
        count = (targets != -100).sum().to(torch.float32)
        losses = []
        for flag, model in (("1", fused_model), ("0", plain_model)):
            os.environ["ABACUS_TP_FUSED"] = flag
            model.zero_grad()
            loss = model(tokens.clamp(min=0), targets=targets, normalizer=count)
            loss.backward()
            losses.append(loss.detach())
        os.environ["ABACUS_TP_FUSED"] = "1"
        torch.cuda.synchronize()
        check_status()
        torch.testing.assert_close(losses[0], losses[1], rtol=1e-5, atol=1e-6)
        for (name, a), b in zip(fused_model.named_parameters(), plain_model.parameters()):
            scale = b.grad.abs().max().clamp(min=1e-12)
            err = ((a.grad - b.grad).abs().max() / scale).item()
            assert err < 2e-4, (name, err)
    # Full training steps through the public Trainer on the fused path.
    fused = Trainer(fused_model, None, device=device)
    plain = Trainer(plain_model, None, device=device)
    for tokens in batches:
        os.environ["ABACUS_TP_FUSED"] = "1"
        loss_f, _ = fused.step(tokens.to(device))
        os.environ["ABACUS_TP_FUSED"] = "0"
        loss_p, _ = plain.step(tokens.to(device))
        os.environ["ABACUS_TP_FUSED"] = "1"
        torch.cuda.synchronize()
        check_status()
        torch.testing.assert_close(loss_f, loss_p, rtol=2e-3, atol=1e-4)
    assert tp_fused._WORKSPACES, "the fused path did not run"
    torch.cuda.synchronize()
    tp_fused.reset()


def test_tp_sp_fused_matches_nccl_path():
    run_ranks(_check, 2, timeout_s=60, backend="nccl")
