"""GPT whose every block is a mixture of experts (``abacus/transformer_moe.py``,
``abacus/transformer_block.py:64-110``).

Attention is never tensor parallel here; expert parallelism forbids dropout
because every rank must keep identical replicated activations. Options beyond
the reference (router type, capacity factor, aux-loss coefficient, EP over
data-parallel ranks) default to the reference's behaviour.
"""
from __future__ import annotations

import torch

from abacus_b200.models.attention import MultiHeadAttention
from abacus_b200.models.layers import Embedding, RMSNorm, Rotary
from abacus_b200.models.moe import MoE, MoEExpertParallel
from abacus_b200.models.transformer import _head
from abacus_b200.parallel import mesh


class TransformerBlockMoe(torch.nn.Module):
    def __init__(
        self,
        dim: int,
        n_heads: int,
        head_dim: int,
        n_experts: int,
        top_k: int,
        dropout: float = 0.0,
        hidden_dim: int | None = None,
        bias_update_speed: float = 1e-3,
        route_scale: float = 1.0,
        expert_parallel: bool = False,
        router: str = "sigmoid",
        capacity_factor: float | None = None,
        aux_loss_coeff: float = 1e-2,
        expert_data_parallel: bool = False,
    ):
        super().__init__()
        _, world_size = mesh.rank_and_world_size("ep")
        if expert_parallel and dropout > 0 and world_size > 1:
            raise ValueError("expert parallel keeps dropout at 0 so replicated layers stay identical")
        self.dim = dim
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.norm_attention = RMSNorm(dim)
        self.attention = MultiHeadAttention(dim, n_heads, head_dim)
        self.norm_mlp = RMSNorm(dim)
        kwargs = dict(
            hidden_dim=hidden_dim, bias_update_speed=bias_update_speed, route_scale=route_scale, router=router,
            capacity_factor=capacity_factor, aux_loss_coeff=aux_loss_coeff,
        )
        if expert_parallel:
            self.moe = MoEExpertParallel(dim, n_experts, top_k, data_parallel=expert_data_parallel, **kwargs)
        else:
            self.moe = MoE(dim, n_experts, top_k, **kwargs)
        self.dropout = torch.nn.Dropout(dropout)

    def forward(self, x_BLD: torch.Tensor, rotary: torch.nn.Module | None = None) -> torch.Tensor:
        if not (self.training and self.dropout.p > 0):
            x_BLD = self.attention(self.norm_attention(x_BLD), rotary, residual=x_BLD)
            return x_BLD + self.moe(self.norm_mlp(x_BLD))
        x_BLD = x_BLD + self.dropout(self.attention(self.norm_attention(x_BLD), rotary))
        return x_BLD + self.dropout(self.moe(self.norm_mlp(x_BLD)))


class TransformerMoe(torch.nn.Module):
    def __init__(
        self,
        dim: int,
        n_heads: int,
        head_dim: int,
        n_blocks: int,
        vocab_size: int,
        n_experts: int,
        top_k: int,
        dropout: float = 0.0,
        hidden_dim: int | None = None,
        bias_update_speed: float = 1e-3,
        route_scale: float = 1.0,
        expert_parallel: bool = False,
        router: str = "sigmoid",
        capacity_factor: float | None = None,
        aux_loss_coeff: float = 1e-2,
        expert_data_parallel: bool = False,
        init_std: float = 1.0,
    ):
        super().__init__()
        self.dim = dim
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.n_blocks = n_blocks
        self.vocab_size = vocab_size
        self.n_experts = n_experts
        self.top_k = top_k
        self.expert_parallel = expert_parallel
        self.expert_data_parallel = expert_data_parallel
        self.embedding = Embedding(vocab_size, dim, init_std=init_std)
        self.rotary = Rotary(head_dim)
        self.blocks = torch.nn.ModuleList(
            [
                TransformerBlockMoe(
                    dim, n_heads, head_dim, n_experts, top_k, dropout, hidden_dim=hidden_dim,
                    bias_update_speed=bias_update_speed, route_scale=route_scale, expert_parallel=expert_parallel,
                    router=router, capacity_factor=capacity_factor, aux_loss_coeff=aux_loss_coeff,
                    expert_data_parallel=expert_data_parallel,
                )
                for _ in range(n_blocks)
            ]
        )
        self.norm = RMSNorm(dim)
        self.w_D_vocab = torch.nn.Parameter(torch.empty(dim, vocab_size))
        torch.nn.init.xavier_uniform_(self.w_D_vocab)

    def aux_loss(self) -> torch.Tensor | None:
        """Sum of the routers' load-balancing losses from the last forward."""
        losses = [b.moe.router.aux_loss for b in self.blocks if b.moe.router.aux_loss is not None]
        return torch.stack(losses).sum() if losses else None

    def hidden_states(self, tokens_BL: torch.Tensor) -> torch.Tensor:
        x_BLD = self.embedding(tokens_BL)
        for block in self.blocks:
            x_BLD = block(x_BLD, self.rotary)
        return self.norm(x_BLD)

    def forward(self, tokens_BL: torch.Tensor, targets=None, normalizer=None) -> torch.Tensor:
        """Logits (B, L, V); with ``targets`` (B, L) the scalar cross-entropy loss."""
        return _head(self.hidden_states(tokens_BL), self.w_D_vocab, targets, normalizer)
