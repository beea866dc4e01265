"""Model layers: RMSNorm, Rotary, Embedding, SwiGLU MLP (+ tensor parallel).

Parameter names, shapes and initialisation match the reference so that a
``state_dict`` moves between the two frameworks unchanged:

* ``RMSNorm.w_gamma_D`` (D,), ones (``abacus/norm.py:13-20``)
* ``Rotary.inv_freq`` (K/2,) buffer (``abacus/rope.py:10-17``)
* ``Embedding.w_vocab_D`` (V, D), normal std 1 (``abacus/embedding.py:11-16``)
* ``MLP.w_gate_DM / w_up_DM`` (D, M), ``w_down_MD`` (M, D), xavier-uniform
  (``abacus/mlp.py:18-28``); the TP variant initialises the full matrices and
  keeps this rank's slice (``abacus/mlp.py:41-63``).
"""
from __future__ import annotations

import torch

from abacus_b200.ops import embedding as embedding_ops
from abacus_b200.ops import gemm
from abacus_b200.ops.norm import rmsnorm
from abacus_b200.parallel import mesh, tp_fused
from abacus_b200.parallel.tensor_parallel import (
    _AllReduceGrads,
    _GatherFromSequenceParallel,
    _ReduceScatterToSequenceParallel,
    _SumOutputs,
)


class RMSNorm(torch.nn.Module):
    """``gamma * x / sqrt(mean(x^2) + 1e-5)``.

    ``sync_grads`` all-reduces gamma's gradient over ``sync_dim`` when each
    rank sees only some tokens (sequence parallel) or heads (tensor parallel).
    """

    def __init__(self, dim: int, sequence_parallel: bool = False, sync_grads: bool = False, sync_dim: str = "tp"):
        super().__init__()
        self.dim = dim
        self.sequence_parallel = sequence_parallel
        self.sync_grads = sequence_parallel or sync_grads
        self.sync_dim = sync_dim
        self.world_size = mesh.rank_and_world_size(sync_dim)[1] if self.sync_grads else 1
        self.w_gamma_D = torch.nn.Parameter(torch.ones(self.dim))

    def gamma(self) -> torch.Tensor:
        if self.sync_grads and self.world_size > 1:
            return _AllReduceGrads.apply(self.w_gamma_D, self.sync_dim)
        return self.w_gamma_D

    def forward(self, x_BLD: torch.Tensor) -> torch.Tensor:
        return rmsnorm(x_BLD, self.gamma())


class Rotary(torch.nn.Module):
    """Non-interleaved rotate-half RoPE, ``inv_freq = base^(-2i/K)``."""

    def __init__(self, dim: int, base: float = 10000):
        super().__init__()
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim))
        self.register_buffer("inv_freq", inv_freq)
        self.seq_len_cached = None
        self.cos_cached = None
        self.sin_cached = None

    def forward(self, x: torch.Tensor, seq_dim: int = 2, positions: torch.Tensor | None = None):
        """cos, sin of shape (1, 1, L, K) for ``x``'s sequence (or ``positions``)."""
        if positions is not None:
            return self._angles(x, positions)
        seq_len = x.shape[seq_dim]
        if seq_len != self.seq_len_cached or self.cos_cached.device != x.device:
            self.seq_len_cached = seq_len
            self.cos_cached, self.sin_cached = self._angles(x, torch.arange(seq_len, device=x.device))
        return self.cos_cached, self.sin_cached

    def _angles(self, x: torch.Tensor, positions: torch.Tensor):
        t = positions.to(device=x.device).type_as(self.inv_freq)
        freqs = torch.einsum("i,j->ij", t, self.inv_freq)
        emb = torch.cat((freqs, freqs), dim=-1).to(x.device)
        return emb.cos()[None, None, :, :], emb.sin()[None, None, :, :]


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2 :]
    return torch.cat((-x2, x1), dim=-1)


def apply_rotary_pos_emb(q, k, cos, sin):
    return (q * cos) + (rotate_half(q) * sin), (k * cos) + (rotate_half(k) * sin)


class Embedding(torch.nn.Module):
    def __init__(self, vocab_size: int, dim: int, init_std: float = 1.0):
        super().__init__()
        self.vocab_size = vocab_size
        self.dim = dim
        self.w_vocab_D = torch.nn.Parameter(torch.empty(vocab_size, dim))
        torch.nn.init.normal_(self.w_vocab_D, std=init_std)

    def forward(self, tokens_BL: torch.Tensor) -> torch.Tensor:
        return embedding_ops.embedding(tokens_BL, self.w_vocab_D)


class MLP(torch.nn.Module):
    """SwiGLU: ``(silu(x @ Wg) * (x @ Wu)) @ Wd``."""

    def __init__(self, dim: int, hidden_dim: int | None = None):
        super().__init__()
        self.dim = dim
        self.hidden_dim = dim if hidden_dim is None else hidden_dim
        self.w_gate_DM = torch.nn.Parameter(torch.empty(self.dim, self.hidden_dim))
        self.w_up_DM = torch.nn.Parameter(torch.empty(self.dim, self.hidden_dim))
        self.w_down_MD = torch.nn.Parameter(torch.empty(self.hidden_dim, self.dim))
        torch.nn.init.xavier_uniform_(self.w_gate_DM)
        torch.nn.init.xavier_uniform_(self.w_up_DM)
        torch.nn.init.xavier_uniform_(self.w_down_MD)

    def forward(self, x_BLD: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """``residual`` (optional) is added in the down-projection's epilogue."""
        return gemm.swiglu_mlp(x_BLD, self.w_gate_DM, self.w_up_DM, self.w_down_MD, residual)


class MLPTensorParallel(torch.nn.Module):
    """Column-parallel gate/up, row-parallel down (Megatron), optional SP."""

    def __init__(self, dim: int, hidden_dim: int | None = None, sequence_parallel: bool = False, dim_name: str = "tp"):
        super().__init__()
        self.dim = dim
        self.hidden_dim = dim if hidden_dim is None else hidden_dim
        self.sequence_parallel = sequence_parallel
        self.dim_name = dim_name
        self.rank, self.world_size = mesh.rank_and_world_size(dim_name)
        if self.hidden_dim % self.world_size != 0:
            raise ValueError(f"MLP hidden dim {self.hidden_dim} is not divisible by world size {self.world_size}")
        local_hidden = self.hidden_dim // self.world_size
        gate_DM = torch.empty(self.dim, self.hidden_dim)
        up_DM = torch.empty(self.dim, self.hidden_dim)
        down_MD = torch.empty(self.hidden_dim, self.dim)
        torch.nn.init.xavier_uniform_(gate_DM)
        torch.nn.init.xavier_uniform_(up_DM)
        torch.nn.init.xavier_uniform_(down_MD)
        start = self.rank * local_hidden
        self.w_gate_DM = torch.nn.Parameter(gate_DM[:, start : start + local_hidden].clone())
        self.w_up_DM = torch.nn.Parameter(up_DM[:, start : start + local_hidden].clone())
        self.w_down_MD = torch.nn.Parameter(down_MD[start : start + local_hidden].clone())
        self._tp_key = tp_fused.new_key("mlp") if sequence_parallel else None

    def forward(self, x_BLD: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """Partial-sum-free output (B, l or L, D); ``residual`` is added when given."""
        if (residual is not None and self.world_size > 1 and self.sequence_parallel
                and (self.hidden_dim // self.world_size) % 32 == 0 and tp_fused.usable(x_BLD, x_BLD.shape[1], self.dim_name)):
            # Gather fused into the gate/up GEMM, reduce-scatter fused into the
            # down GEMM's epilogue, residual added in the reduction.
            return tp_fused.swiglu(x_BLD, self.w_gate_DM, self.w_up_DM, self.w_down_MD, residual, self._tp_key,
                                   self.dim_name)
        out = self._forward_unfused(x_BLD)
        return out if residual is None else residual + out

    def _forward_unfused(self, x_BLD: torch.Tensor) -> torch.Tensor:
        if self.world_size > 1 and self.sequence_parallel:
            x_BLD = _GatherFromSequenceParallel.apply(x_BLD, self.dim_name)
        elif self.world_size > 1:
            x_BLD = _AllReduceGrads.apply(x_BLD, self.dim_name)
        partial_BLD = gemm.swiglu_mlp(x_BLD, self.w_gate_DM, self.w_up_DM, self.w_down_MD)
        if self.world_size > 1 and self.sequence_parallel:
            return _ReduceScatterToSequenceParallel.apply(partial_BLD, self.dim_name)
        if self.world_size > 1:
            return _SumOutputs.apply(partial_BLD, self.dim_name)
        return partial_BLD
