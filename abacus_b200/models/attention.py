"""Multi-head attention with QK-norm + RoPE, tensor/sequence/context parallel.

Parameters (``abacus/attention.py:69-115``): ``w_q_DHK``, ``w_k_DHK``,
``w_v_DHK`` (D, H, K), ``w_o_HKD`` (H, K, D), xavier-uniform on the
``d (h k)`` / ``(h k) d`` views, TP slices taken from the full init; QK-norm
gammas ``q_norm`` / ``k_norm`` (K,).

CUDA path per call: one N-segmented QKV GEMM -> QK-norm + RoPE kernel ->
tcgen05 flash attention -> O-projection GEMM with the residual add in its
epilogue. Context parallel all-gathers the rotated K and V (token-major, so
no permute copies) and masks by global zigzag positions inside the kernel.
CPU path: the reference's materialised formulation.

Deliberate fix versus the reference: under context parallelism the QK-norm
gamma gradients are summed once (by the trainer's CP gradient sum,
``abacus/distributed/context_parallel.py:56-66``); the reference also
all-reduces them in the forward (``abacus/attention.py:113-115``), which
sums them twice.
"""
from __future__ import annotations

import torch

from abacus_b200.models.layers import RMSNorm, Rotary, apply_rotary_pos_emb
from abacus_b200.ops import attention as attn_ops
from abacus_b200.ops import gemm
from abacus_b200.parallel import cp_fused, mesh, tp_fused
from abacus_b200.parallel.context_parallel import (
    _AllGatherSequenceBlock,
    all_gather_positions,
    zigzag_positions,
)
from abacus_b200.parallel.tensor_parallel import (
    _AllReduceGrads,
    _GatherFromSequenceParallel,
    _ReduceScatterToSequenceParallel,
    _SumOutputs,
)


def _later_than_query(query_positions: torch.Tensor, key_positions: torch.Tensor) -> torch.Tensor:
    """True where a key is strictly after its query (masked out)."""
    return query_positions[:, None] < key_positions[None, :]


class ScaledDotProductAttention(torch.nn.Module):
    """Single-head causal attention with (D, D) weights (``abacus/attention.py:33-64``)."""

    def __init__(self, dim: int):
        super().__init__()
        self.dim = dim
        self.w_q_DD = torch.nn.Parameter(torch.empty(dim, dim))
        self.w_k_DD = torch.nn.Parameter(torch.empty(dim, dim))
        self.w_v_DD = torch.nn.Parameter(torch.empty(dim, dim))
        torch.nn.init.xavier_uniform_(self.w_q_DD)
        torch.nn.init.xavier_uniform_(self.w_k_DD)
        torch.nn.init.xavier_uniform_(self.w_v_DD)

    def forward(self, q_BLD, k_BLD, v_BLD):
        q_BLD = q_BLD @ self.w_q_DD
        k_BLD = k_BLD @ self.w_k_DD
        v_BLD = v_BLD @ self.w_v_DD
        scores = torch.matmul(q_BLD, k_BLD.transpose(-2, -1)) / (self.dim**0.5)
        qp = torch.arange(q_BLD.shape[1], device=q_BLD.device)
        kp = torch.arange(k_BLD.shape[1], device=k_BLD.device)
        scores = scores.masked_fill(_later_than_query(qp, kp), float("-inf"))
        return torch.matmul(torch.softmax(scores, dim=-1), v_BLD)


class MultiHeadAttention(torch.nn.Module):
    def __init__(
        self,
        dim: int,
        n_heads: int,
        head_dim: int,
        tensor_parallel: bool = False,
        sequence_parallel: bool = False,
        context_parallel: bool = False,
    ):
        super().__init__()
        if sequence_parallel and not tensor_parallel:
            raise ValueError("sequence_parallel requires tensor_parallel")
        if context_parallel and (tensor_parallel or sequence_parallel):
            raise ValueError("context_parallel does not combine with tensor or sequence parallel")
        self.dim = dim
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.tensor_parallel = tensor_parallel
        self.sequence_parallel = sequence_parallel
        self.context_parallel = context_parallel
        if tensor_parallel:
            self.rank, self.world_size = mesh.rank_and_world_size("tp")
            if n_heads % self.world_size != 0:
                raise ValueError(f"n_heads {n_heads} is not divisible by world size {self.world_size}")
        else:
            self.rank, self.world_size = 0, 1
        self.local_heads = n_heads // self.world_size
        q_DHK = torch.empty(dim, n_heads, head_dim)
        k_DHK = torch.empty(dim, n_heads, head_dim)
        v_DHK = torch.empty(dim, n_heads, head_dim)
        o_HKD = torch.empty(n_heads, head_dim, dim)
        torch.nn.init.xavier_uniform_(q_DHK.view(dim, n_heads * head_dim))
        torch.nn.init.xavier_uniform_(k_DHK.view(dim, n_heads * head_dim))
        torch.nn.init.xavier_uniform_(v_DHK.view(dim, n_heads * head_dim))
        torch.nn.init.xavier_uniform_(o_HKD.view(n_heads * head_dim, dim))
        start = self.rank * self.local_heads
        self.w_q_DHK = torch.nn.Parameter(q_DHK[:, start : start + self.local_heads].clone())
        self.w_k_DHK = torch.nn.Parameter(k_DHK[:, start : start + self.local_heads].clone())
        self.w_v_DHK = torch.nn.Parameter(v_DHK[:, start : start + self.local_heads].clone())
        self.w_o_HKD = torch.nn.Parameter(o_HKD[start : start + self.local_heads].clone())
        self._tp_key = tp_fused.new_key("attn") if tensor_parallel and sequence_parallel else None
        self._cp_key = tp_fused.new_key("cpattn") if context_parallel else None
        # One gamma shared by all heads; summed over TP ranks (heads sharded).
        self.q_norm = RMSNorm(head_dim, sync_grads=tensor_parallel)
        self.k_norm = RMSNorm(head_dim, sync_grads=tensor_parallel)

    # ------------------------------------------------------------------ API
    def forward(self, x_BLD: torch.Tensor, rotary: Rotary | None = None, residual: torch.Tensor | None = None):
        """Attention output (B, L, D); ``residual`` is added when given (fused
        into the O-projection epilogue on one rank)."""
        if self.context_parallel:
            return self._forward_context_parallel(x_BLD, rotary, residual)
        if self._tp_fused_usable(x_BLD, rotary, residual):
            return self._forward_tp_fused(x_BLD, rotary, residual)
        if self.world_size > 1 and self.sequence_parallel:
            x_BLD = _GatherFromSequenceParallel.apply(x_BLD, "tp")
        elif self.world_size > 1:
            x_BLD = _AllReduceGrads.apply(x_BLD, "tp")
        fuse_residual = residual is not None and self.world_size == 1
        if x_BLD.is_cuda and rotary is not None:
            out = self._forward_fused(x_BLD, rotary, residual if fuse_residual else None)
        else:
            out = self._forward_reference(x_BLD, rotary)
            if fuse_residual:
                out = residual + out
        if self.world_size > 1 and self.sequence_parallel:
            out = _ReduceScatterToSequenceParallel.apply(out, "tp")
        elif self.world_size > 1:
            out = _SumOutputs.apply(out, "tp")
        if residual is not None and not fuse_residual:
            out = residual + out
        return out

    def _tp_fused_usable(self, x_BLD, rotary, residual) -> bool:
        return (self.world_size > 1 and self.sequence_parallel and residual is not None and rotary is not None
                and (self.local_heads * self.head_dim) % 128 == 0 and tp_fused.usable(x_BLD, x_BLD.shape[1]))

    def _forward_tp_fused(self, x_BLD, rotary, residual):
        """SP shard -> (gather fused into the QKV GEMM) -> attention on the local
        heads -> (O-projection GEMM scattering its rows to their owners) ->
        residual + reduce, all over NVLink peer memory."""
        b = x_BLD.shape[0]
        qkv = tp_fused.gather_qkv(x_BLD, self.w_q_DHK, self.w_k_DHK, self.w_v_DHK, self._tp_key)
        o = attn_ops.causal_attention(
            qkv, b, self.local_heads, self.head_dim, self.q_norm.gamma(), self.k_norm.gamma(), rotary.inv_freq
        )
        w_o = self.w_o_HKD.reshape(self.local_heads * self.head_dim, self.dim)
        return tp_fused.row_scatter(o, w_o, residual, self._tp_key)

    def _forward_fused(self, x_BLD, rotary, residual):
        b, length, _ = x_BLD.shape
        o = attn_ops.qkv_attention(x_BLD, self.w_q_DHK, self.w_k_DHK, self.w_v_DHK, b, self.local_heads,
                                   self.head_dim, self.q_norm.gamma(), self.k_norm.gamma(), rotary.inv_freq)
        w_o = self.w_o_HKD.reshape(self.local_heads * self.head_dim, self.dim)
        res2 = None if residual is None else residual.reshape(-1, self.dim)
        return gemm.linear(o, w_o, res2).view(b, length, self.dim)

    def _forward_reference(self, x_BLD, rotary):
        q_BHLK = self._split_heads(x_BLD, self.w_q_DHK)
        k_BHLK = self._split_heads(x_BLD, self.w_k_DHK)
        v_BHLK = self._split_heads(x_BLD, self.w_v_DHK)
        q_BHLK, k_BHLK = self._normalize_qk(q_BHLK, k_BHLK)
        if rotary is not None:
            q_BHLK, k_BHLK = self._apply_rope(q_BHLK, k_BHLK, rotary)
        scores = torch.einsum("bhlk,bhsk->bhls", q_BHLK, k_BHLK) / (self.head_dim**0.5)
        positions = torch.arange(q_BHLK.shape[2], device=q_BHLK.device)
        scores = scores.masked_fill(_later_than_query(positions, positions), float("-inf"))
        out_BHLK = torch.einsum("bhls,bhsk->bhlk", torch.softmax(scores, dim=-1), v_BHLK)
        return self._merge_heads(out_BHLK) @ self.w_o_HKD.reshape(-1, self.dim)

    def _forward_context_parallel(self, x_BLD, rotary, residual):
        rank, world = mesh.rank_and_world_size("cp")
        b, local_len, _ = x_BLD.shape
        positions = zigzag_positions(local_len * world, rank, world).to(x_BLD.device)
        if x_BLD.is_cuda and rotary is not None:
            qkv = gemm.qkv_projection(x_BLD, self.w_q_DHK, self.w_k_DHK, self.w_v_DHK)
            token_pos = positions.repeat(b)
            q, k, v = attn_ops.qk_prologue(
                qkv, self.local_heads, self.head_dim, self.q_norm.w_gamma_D, self.k_norm.w_gamma_D,
                rotary.inv_freq, local_len, positions=token_pos, n_positions=local_len * world,
            )
            hk = self.local_heads * self.head_dim
            k_pos = all_gather_positions(positions)
            if world > 1 and cp_fused.usable(x_BLD, local_len, self.head_dim):
                # K/V gather fused into the flash kernel's loads, dK/dV
                # reduce-scatter into its backward stores (NVLink peer memory).
                o = cp_fused.attention(q, k, v, b, self.local_heads, self.head_dim, positions, k_pos, self._cp_key)
            else:
                k = _GatherFromSequenceParallel.apply(k.view(b, local_len, hk), "cp").reshape(-1, hk)
                v = _GatherFromSequenceParallel.apply(v.reshape(b, local_len, hk), "cp").reshape(-1, hk)
                o = attn_ops.flash_attention(q, k, v, b, self.local_heads, self.head_dim, q_pos=positions,
                                             k_pos=k_pos)
            w_o = self.w_o_HKD.reshape(hk, self.dim)
            res2 = None if residual is None else residual.reshape(-1, self.dim)
            return gemm.linear(o, w_o, res2).view(b, local_len, self.dim)
        q_BHLK = self._split_heads(x_BLD, self.w_q_DHK)
        k_BHLK = self._split_heads(x_BLD, self.w_k_DHK)
        v_BHLK = self._split_heads(x_BLD, self.w_v_DHK)
        q_BHLK, k_BHLK = self._normalize_qk(q_BHLK, k_BHLK)
        if rotary is not None:
            q_BHLK, k_BHLK = self._apply_rope(q_BHLK, k_BHLK, rotary, positions)
        out_BHLK = self._attend_blocks(q_BHLK, k_BHLK, v_BHLK, positions)
        out = self._merge_heads(out_BHLK) @ self.w_o_HKD.reshape(-1, self.dim)
        return out if residual is None else residual + out

    def _attend_blocks(self, q_BHLK, k_BHLK, v_BHLK, positions):
        k_BHLK = _AllGatherSequenceBlock.apply(k_BHLK)
        v_BHLK = _AllGatherSequenceBlock.apply(v_BHLK)
        key_positions = all_gather_positions(positions)
        scores = torch.einsum("bhlk,bhsk->bhls", q_BHLK, k_BHLK) / (self.head_dim**0.5)
        scores = scores.masked_fill(_later_than_query(positions, key_positions), float("-inf"))
        return torch.einsum("bhls,bhsk->bhlk", torch.softmax(scores, dim=-1), v_BHLK)

    def _normalize_qk(self, q_BHLK, k_BHLK):
        """RMSNorm over the head dimension, before RoPE."""
        return self.q_norm(q_BHLK), self.k_norm(k_BHLK)

    def _apply_rope(self, q_BHLK, k_BHLK, rotary, positions=None):
        cos, sin = rotary(q_BHLK, seq_dim=2, positions=positions)
        return apply_rotary_pos_emb(q_BHLK, k_BHLK, cos, sin)

    def _split_heads(self, x_BLD, w_DHK):
        b, length, _ = x_BLD.shape
        projected = x_BLD @ w_DHK.reshape(w_DHK.shape[0], -1)
        return projected.view(b, length, self.local_heads, self.head_dim).transpose(1, 2)

    def _merge_heads(self, out_BHLK):
        b, h, length, k = out_BHLK.shape
        return out_BHLK.transpose(1, 2).reshape(b, length, h * k)
