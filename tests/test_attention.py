"""Attention semantics: QK-norm before RoPE, causal softmax (CPU oracle path)."""
import torch
import torch.nn.functional as F

from abacus_b200.attention import MultiHeadAttention, ScaledDotProductAttention
from abacus_b200.rope import Rotary


def test_legacy_single_head_attention_is_causal_sdpa():
    torch.manual_seed(0)
    att = ScaledDotProductAttention(6)
    q, k, v = torch.randn(2, 5, 6), torch.randn(2, 5, 6), torch.randn(2, 5, 6)
    expected = F.scaled_dot_product_attention(q @ att.w_q_DD, k @ att.w_k_DD, v @ att.w_v_DD, is_causal=True)
    torch.testing.assert_close(att(q, k, v), expected)


def _manual(att, x, rotary, positions=None):
    b, length, d = x.shape
    h, kd = att.local_heads, att.head_dim

    def heads(w):
        return (x @ w.reshape(d, -1)).view(b, length, h, kd).transpose(1, 2)

    q = att.q_norm(heads(att.w_q_DHK))
    k = att.k_norm(heads(att.w_k_DHK))
    v = heads(att.w_v_DHK)
    cos, sin = rotary(q, seq_dim=2, positions=positions)
    rot = lambda t: torch.cat((-t[..., kd // 2 :], t[..., : kd // 2]), -1)  # noqa: E731
    q, k = q * cos + rot(q) * sin, k * cos + rot(k) * sin
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    return o.transpose(1, 2).reshape(b, length, h * kd) @ att.w_o_HKD.reshape(h * kd, d)


def test_mha_normalizes_before_rope_and_is_causal():
    torch.manual_seed(1)
    att = MultiHeadAttention(8, 2, 4)
    with torch.no_grad():
        att.q_norm.w_gamma_D.uniform_(0.5, 1.5)
        att.k_norm.w_gamma_D.uniform_(0.5, 1.5)
    rot = Rotary(4)
    x = torch.randn(2, 6, 8)
    torch.testing.assert_close(att(x, rot), _manual(att, x, rot))


def test_mha_residual_argument():
    torch.manual_seed(2)
    att = MultiHeadAttention(8, 2, 4)
    rot = Rotary(4)
    x, r = torch.randn(1, 5, 8), torch.randn(1, 5, 8)
    torch.testing.assert_close(att(x, rot, residual=r), r + att(x, rot))


def test_context_parallel_path_on_one_rank_matches_causal():
    torch.manual_seed(3)
    att = MultiHeadAttention(8, 2, 4, context_parallel=True)
    with torch.no_grad():
        att.q_norm.w_gamma_D.uniform_(0.5, 1.5)
    rot = Rotary(4)
    x = torch.randn(2, 4, 8)
    torch.testing.assert_close(att(x, rot), _manual(att, x, rot))


def test_parameter_layout_matches_reference_names():
    att = MultiHeadAttention(12, 3, 4)
    shapes = {n: tuple(p.shape) for n, p in att.named_parameters()}
    assert shapes == {
        "w_q_DHK": (12, 3, 4), "w_k_DHK": (12, 3, 4), "w_v_DHK": (12, 3, 4), "w_o_HKD": (3, 4, 12),
        "q_norm.w_gamma_D": (4,), "k_norm.w_gamma_D": (4,),
    }
