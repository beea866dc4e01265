"""Dense GPT: blocks, Transformer and PipelineStage.

Structure and parameter layout follow ``abacus/transformer_block.py:18-61``
and ``abacus/transformer.py``: pre-norm blocks ``x + drop(attn(norm(x)))``,
``x + drop(mlp(norm(x)))``; embedding -> blocks -> final RMSNorm -> untied
``w_D_vocab`` (D, V) logits; PipelineStage keeps an even slice of blocks with
*local* indices, the embedding on rank 0 and norm + logits on the last rank.

Additions (all default to the reference's behaviour): ``hidden_dim`` (the
reference hard-codes 4*dim), ``init_std`` for the embedding (reference: 1.0),
and ``context_parallel`` on PipelineStage for the CP x PP mesh.

On CUDA the residual adds are fused into the O-projection and
down-projection epilogues when dropout is inactive.
"""
from __future__ import annotations

import torch

from abacus_b200.models.attention import MultiHeadAttention
from abacus_b200.models.layers import MLP, Embedding, MLPTensorParallel, RMSNorm, Rotary
from abacus_b200.ops import gemm
from abacus_b200.ops.cross_entropy import fused_linear_cross_entropy
from abacus_b200.parallel import cp_fused, mesh, tp_fused
from abacus_b200.parallel.context_parallel import zigzag_positions
from abacus_b200.parallel.tensor_parallel import (
    _AllReduceGrads,
    _GatherReplicated,
    _ScatterToSequenceParallel,
    _SumOutputs,
)


class TransformerBlock(torch.nn.Module):
    def __init__(
        self,
        dim: int,
        n_heads: int,
        head_dim: int,
        dropout: float = 0.0,
        tensor_parallel: bool = False,
        sequence_parallel: bool = False,
        context_parallel: bool = False,
        hidden_dim: int | None = None,
    ):
        super().__init__()
        if sequence_parallel and not tensor_parallel:
            raise ValueError("sequence_parallel requires tensor_parallel")
        if context_parallel and (tensor_parallel or sequence_parallel):
            raise ValueError("context_parallel does not combine with tensor or sequence parallel")
        self.dim = dim
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.hidden_dim = 4 * dim if hidden_dim is None else hidden_dim
        self.norm_attention = RMSNorm(dim, sequence_parallel)
        self.attention = MultiHeadAttention(dim, n_heads, head_dim, tensor_parallel, sequence_parallel, context_parallel)
        self.norm_mlp = RMSNorm(dim, sequence_parallel)
        if tensor_parallel:
            self.mlp = MLPTensorParallel(dim, hidden_dim=self.hidden_dim, sequence_parallel=sequence_parallel)
        else:
            self.mlp = MLP(dim, hidden_dim=self.hidden_dim)
        self.dropout = torch.nn.Dropout(dropout)

    def _dropout_active(self) -> bool:
        return self.training and self.dropout.p > 0

    def forward(self, x_BLD: torch.Tensor, rotary: torch.nn.Module | None = None) -> torch.Tensor:
        if not self._dropout_active():
            x_BLD = self.attention(self.norm_attention(x_BLD), rotary, residual=x_BLD)
            return self.mlp(self.norm_mlp(x_BLD), residual=x_BLD)
        x_BLD = x_BLD + self.dropout(self.attention(self.norm_attention(x_BLD), rotary))
        return x_BLD + self.dropout(self.mlp(self.norm_mlp(x_BLD)))


def _logits(x_BLD: torch.Tensor, w_D_vocab: torch.Tensor) -> torch.Tensor:
    return gemm.linear(x_BLD, w_D_vocab)


def _head(x_BLD, w_D_vocab, targets, normalizer):
    """Logits, or (with ``targets``) the fused linear + cross-entropy loss
    ``sum CE / normalizer`` (normalizer defaults to the target count)."""
    if targets is None:
        return _logits(x_BLD, w_D_vocab)
    return fused_linear_cross_entropy(x_BLD, w_D_vocab, targets, normalizer)


class Transformer(torch.nn.Module):
    def __init__(
        self,
        dim: int,
        n_heads: int,
        head_dim: int,
        n_blocks: int,
        vocab_size: int,
        dropout: float = 0.0,
        tensor_parallel: bool = False,
        sequence_parallel: bool = False,
        context_parallel: bool = False,
        hidden_dim: int | None = None,
        init_std: float = 1.0,
    ):
        super().__init__()
        if sequence_parallel and not tensor_parallel:
            raise ValueError("sequence_parallel requires tensor_parallel")
        if context_parallel and (tensor_parallel or sequence_parallel):
            raise ValueError("context_parallel does not combine with tensor or sequence parallel")
        self.dim = dim
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.n_blocks = n_blocks
        self.vocab_size = vocab_size
        self.sequence_parallel = sequence_parallel
        self.context_parallel = context_parallel
        self.tensor_parallel = tensor_parallel
        _, self.world_size = mesh.rank_and_world_size("tp") if sequence_parallel else (0, 1)
        self.embedding = Embedding(vocab_size, dim, init_std=init_std)
        self.rotary = Rotary(head_dim)
        self.blocks = torch.nn.ModuleList(
            [
                TransformerBlock(
                    dim, n_heads, head_dim, dropout, tensor_parallel, sequence_parallel, context_parallel, hidden_dim
                )
                for _ in range(n_blocks)
            ]
        )
        self.norm = RMSNorm(dim, sequence_parallel)
        self.w_D_vocab = torch.nn.Parameter(torch.empty(dim, vocab_size))
        torch.nn.init.xavier_uniform_(self.w_D_vocab)

    def hidden_states(self, tokens_BL: torch.Tensor) -> torch.Tensor:
        """Final-norm output (B, L, D) (replicated over SP ranks)."""
        x_BLD = self._final_norm(tokens_BL)
        if self.sequence_parallel and self.world_size > 1:
            x_BLD = _GatherReplicated.apply(x_BLD, "tp")
        return x_BLD

    def _final_norm(self, tokens_BL: torch.Tensor) -> torch.Tensor:
        """Final-norm output: (B, L, D), or this rank's (B, L/P, D) shard under SP."""
        if self.sequence_parallel and self.world_size > 1:
            length = tokens_BL.shape[1]
            if length % self.world_size != 0:
                raise ValueError(f"sequence length {length} is not divisible by world size {self.world_size}")
        if self.context_parallel:
            rank, world = mesh.rank_and_world_size("cp")
            if world > 1:
                positions = zigzag_positions(tokens_BL.shape[1], rank, world)
                tokens_BL = tokens_BL.index_select(1, positions.to(tokens_BL.device))
                if tokens_BL.is_cuda:
                    cp_fused.begin_step(tokens_BL.device)
        if self.sequence_parallel and self.world_size > 1 and tokens_BL.is_cuda:
            # Fused TP buffers are reused every step: wait (bounded, on the
            # device) until every TP rank finished the previous step.
            tp_fused.begin_step(tokens_BL.device)
        x_BLD = self.embedding(tokens_BL)
        if self.sequence_parallel and self.world_size > 1:
            x_BLD = _ScatterToSequenceParallel.apply(x_BLD, "tp")
        for block in self.blocks:
            x_BLD = block(x_BLD, self.rotary)
        return self.norm(x_BLD)

    def forward(self, tokens_BL: torch.Tensor, targets=None, normalizer=None) -> torch.Tensor:
        """Logits (B, L, V); with ``targets`` (B, L) the scalar training loss.

        Under sequence parallel the loss is computed on each rank's own
        sequence shard (no gather of the final hidden states) and summed over
        the TP group; the head weight's gradient is summed over the group in
        backward. Same value and gradients as the reference's replicated head
        (``abacus/transformer.py:80-97``), 1/P of its work per rank.
        """
        if targets is not None and self.sequence_parallel and self.world_size > 1:
            rank, _ = mesh.rank_and_world_size("tp")
            x_BlD = self._final_norm(tokens_BL)
            chunk = x_BlD.shape[1]
            if normalizer is None:
                normalizer = (targets != -100).sum().to(torch.float32)
            weight = _AllReduceGrads.apply(self.w_D_vocab, "tp")
            partial = _head(x_BlD, weight, targets[:, rank * chunk : (rank + 1) * chunk], normalizer)
            return _SumOutputs.apply(partial, "tp")
        return _head(self.hidden_states(tokens_BL), self.w_D_vocab, targets, normalizer)


class PipelineStage(torch.nn.Module):
    """One pipeline rank: an even slice of blocks, plus the ends on the edge ranks.

    Rank 0 owns the embedding; the last rank owns the final norm and the
    logits. Block indices are local (``abacus/transformer.py:99-159``).
    """

    def __init__(
        self,
        dim: int,
        n_heads: int,
        head_dim: int,
        n_blocks: int,
        vocab_size: int,
        rank: int,
        world_size: int,
        dropout: float = 0.0,
        hidden_dim: int | None = None,
        context_parallel: bool = False,
        init_std: float = 1.0,
    ):
        super().__init__()
        if world_size < 1:
            raise ValueError(f"world_size must be at least 1, got {world_size}")
        if n_blocks < 1:
            raise ValueError(f"n_blocks must be at least 1, got {n_blocks}")
        if n_blocks % world_size != 0:
            raise ValueError(f"n_blocks {n_blocks} is not divisible by world size {world_size}")
        if not 0 <= rank < world_size:
            raise ValueError(f"rank {rank} is outside world size {world_size}")
        self.dim = dim
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.n_blocks = n_blocks
        self.vocab_size = vocab_size
        self.rank = rank
        self.world_size = world_size
        self.context_parallel = context_parallel
        per_rank = n_blocks // world_size
        if rank == 0:
            self.embedding = Embedding(vocab_size, dim, init_std=init_std)
        self.rotary = Rotary(head_dim)
        self.blocks = torch.nn.ModuleList(
            [
                TransformerBlock(dim, n_heads, head_dim, dropout, context_parallel=context_parallel, hidden_dim=hidden_dim)
                for _ in range(per_rank)
            ]
        )
        if rank == world_size - 1:
            self.norm = RMSNorm(dim)
            self.w_D_vocab = torch.nn.Parameter(torch.empty(dim, vocab_size))
            torch.nn.init.xavier_uniform_(self.w_D_vocab)

    @property
    def is_first(self) -> bool:
        return self.rank == 0

    @property
    def is_last(self) -> bool:
        return self.rank == self.world_size - 1

    def hidden_states(self, x: torch.Tensor) -> torch.Tensor:
        if self.rank == 0:
            if self.context_parallel:
                cp_rank, cp_world = mesh.rank_and_world_size("cp")
                if cp_world > 1:
                    positions = zigzag_positions(x.shape[1], cp_rank, cp_world)
                    x = x.index_select(1, positions.to(x.device))
            x = self.embedding(x)
        for block in self.blocks:
            x = block(x, self.rotary)
        if self.is_last:
            x = self.norm(x)
        return x

    def forward(self, x: torch.Tensor, targets=None, normalizer=None) -> torch.Tensor:
        x = self.hidden_states(x)
        if self.is_last:
            return _head(x, self.w_D_vocab, targets, normalizer)
        return x
