"""Layer semantics against PyTorch formulations (CPU)."""
import pytest
import torch

from abacus_b200.embedding import Embedding
from abacus_b200.mlp import MLP
from abacus_b200.norm import RMSNorm
from abacus_b200.rope import Rotary, apply_rotary_pos_emb


def test_rmsnorm_equals_torch_rmsnorm():
    torch.manual_seed(0)
    norm = RMSNorm(6)
    with torch.no_grad():
        norm.w_gamma_D.uniform_(-2, 2)
    ref = torch.nn.RMSNorm(6, eps=1e-5)
    with torch.no_grad():
        ref.weight.copy_(norm.w_gamma_D)
    x = torch.randn(3, 5, 6)
    torch.testing.assert_close(norm(x), ref(x))


def test_mlp_is_swiglu_of_three_linears():
    torch.manual_seed(1)
    mlp = MLP(6, 10)
    x = torch.randn(2, 4, 6)
    g = torch.nn.functional.linear(x, mlp.w_gate_DM.t())
    u = torch.nn.functional.linear(x, mlp.w_up_DM.t())
    expected = torch.nn.functional.linear(torch.nn.functional.silu(g) * u, mlp.w_down_MD.t())
    torch.testing.assert_close(mlp(x), expected)
    assert mlp.w_gate_DM.shape == (6, 10) and mlp.w_down_MD.shape == (10, 6)


def test_mlp_residual_argument_adds_input():
    torch.manual_seed(2)
    mlp = MLP(4, 8)
    x, r = torch.randn(2, 3, 4), torch.randn(2, 3, 4)
    torch.testing.assert_close(mlp(x, residual=r), r + mlp(x))


def test_rotary_is_rotate_half_with_base_10000():
    rot = Rotary(8)
    torch.testing.assert_close(rot.inv_freq, 1.0 / 10000 ** (torch.arange(0, 8, 2).float() / 8))
    q = torch.randn(1, 2, 5, 8)
    k = torch.randn(1, 2, 5, 8)
    cos, sin = rot(q, seq_dim=2)
    assert cos.shape == (1, 1, 5, 8)
    q2, k2 = apply_rotary_pos_emb(q, k, cos, sin)
    # Position p rotates the pair (i, i + 4) by angle p * inv_freq[i].
    p, i = 3, 1
    ang = p * rot.inv_freq[i]
    a, b = q[0, 0, p, i], q[0, 0, p, i + 4]
    torch.testing.assert_close(q2[0, 0, p, i], a * torch.cos(ang) - b * torch.sin(ang))
    torch.testing.assert_close(q2[0, 0, p, i + 4], b * torch.cos(ang) + a * torch.sin(ang))
    # Norm-preserving.
    torch.testing.assert_close(q2.norm(dim=-1), q.norm(dim=-1))


def test_rotary_explicit_positions():
    rot = Rotary(4)
    x = torch.zeros(1, 1, 3, 4)
    cos, sin = rot(x, positions=torch.tensor([7, 2, 9]))
    full_cos, _ = rot(torch.zeros(1, 1, 10, 4))
    torch.testing.assert_close(cos[0, 0], full_cos[0, 0, [7, 2, 9]])


@pytest.mark.parametrize("std", [1.0, 0.02])
def test_embedding_init_and_lookup(std):
    torch.manual_seed(3)
    emb = Embedding(4000, 64, init_std=std)
    assert abs(emb.w_vocab_D.std().item() - std) < 0.05 * std
    tok = torch.tensor([[3, 1], [0, 3]])
    torch.testing.assert_close(emb(tok), emb.w_vocab_D[tok])
