"""Causal multi-head attention core with the QK-RMSNorm + RoPE prologue.

Input is the fused projection ``qkv`` (T, 3*H*K) in token-major order (rows
``b*L + l``), exactly what the QKV GEMM writes; output is (T, H*K), what the
O-projection GEMM reads. Semantics (``abacus/attention.py:118-150,175-213``):

* q and k are RMS-normalised over head_dim (eps 1e-5, one gamma shared by all
  heads) *before* RoPE;
* RoPE is the non-interleaved rotate-half form with base 10000
  (``abacus/rope.py:31-47``);
* scores are scaled by 1/sqrt(head_dim) and masked where key position >
  query position (global positions under context parallelism).

CUDA: ``qkv_attention`` normalises and rotates q and k in the QKV GEMM's
epilogue (fp32 mode; otherwise a prologue kernel writes them once), then the tcgen05
flash-attention kernels (``csrc/attention``) compute the output without ever
materialising the (L, L) score matrix; backward recomputes the scores tile by
tile. CPU: the reference's materialised formulation.
"""
from __future__ import annotations

import math
import os

import torch

from abacus_b200.ops import gemm, precision
from abacus_b200.ops._ext import ext
from abacus_b200.ops.norm import EPS, rmsnorm_reference


def rope_tables(inv_freq: torch.Tensor, n_positions: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables (P, K/2): angle = position * inv_freq, fp32 (``rope.py:31-35``)."""
    t = torch.arange(n_positions, device=device, dtype=inv_freq.dtype)
    freqs = torch.outer(t, inv_freq.to(device))
    return freqs.cos().contiguous(), freqs.sin().contiguous()


def _rotate_half(x):
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2 :]
    return torch.cat((-x2, x1), dim=-1)


def attention_reference(
    qkv: torch.Tensor,
    batch: int,
    heads: int,
    head_dim: int,
    q_gamma: torch.Tensor,
    k_gamma: torch.Tensor,
    inv_freq: torch.Tensor | None,
    q_positions: torch.Tensor,
    k_positions: torch.Tensor,
    kv: tuple[torch.Tensor, torch.Tensor] | None = None,
) -> torch.Tensor:
    """Materialised attention (the oracle). ``kv`` overrides K/V (already
    normalised and rotated) for context parallelism."""
    t = qkv.shape[0]
    length = t // batch
    hk = heads * head_dim
    q = qkv[:, :hk].reshape(batch, length, heads, head_dim).transpose(1, 2)
    k = qkv[:, hk : 2 * hk].reshape(batch, length, heads, head_dim).transpose(1, 2)
    v = qkv[:, 2 * hk :].reshape(batch, length, heads, head_dim).transpose(1, 2)
    q = rmsnorm_reference(q, q_gamma)
    k = rmsnorm_reference(k, k_gamma)
    if inv_freq is not None:
        qa = torch.outer(q_positions.to(inv_freq.dtype), inv_freq)
        qe = torch.cat((qa, qa), dim=-1)
        q = q * qe.cos() + _rotate_half(q) * qe.sin()
        ka = torch.outer(q_positions.to(inv_freq.dtype), inv_freq)
        ke = torch.cat((ka, ka), dim=-1)
        k = k * ke.cos() + _rotate_half(k) * ke.sin()
    if kv is not None:
        k, v = kv(k, v)
    scores = torch.einsum("bhlk,bhsk->bhls", q, k) / (head_dim**0.5)
    mask = q_positions[:, None] < k_positions[None, :]
    scores = scores.masked_fill(mask.to(scores.device), float("-inf"))
    weights = torch.softmax(scores, dim=-1)
    out = torch.einsum("bhls,bhsk->bhlk", weights, v)
    return out.transpose(1, 2).reshape(t, hk)


class _QKPrologue(torch.autograd.Function):
    """(T, 3HK) raw projections -> rotated q, k (T, HK) each; v is a view."""

    @staticmethod
    def forward(ctx, qkv, q_gamma, k_gamma, cos_t, sin_t, positions, heads, head_dim, seq_len):
        t = qkv.shape[0]
        hk = heads * head_dim
        q = torch.empty(t, hk, device=qkv.device, dtype=torch.float32)
        k = torch.empty_like(q)
        rstd = torch.empty(t * 2 * heads, device=qkv.device, dtype=torch.float32)
        ext().qk_prologue_fwd(qkv, q_gamma, k_gamma, cos_t, sin_t, positions, seq_len, q, k, rstd, heads, head_dim, EPS)
        ctx.save_for_backward(qkv, q_gamma, k_gamma, cos_t, sin_t, positions, rstd)
        ctx.dims = (heads, head_dim, seq_len)
        return q, k, qkv.narrow(1, 2 * hk, hk)

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, q_gamma, k_gamma, cos_t, sin_t, positions, rstd = ctx.saved_tensors
        dqkv, dgq, dgk = _prologue_grads(qkv, q_gamma, k_gamma, cos_t, sin_t, positions, rstd, dq, dk, dv, *ctx.dims)
        return dqkv, dgq, dgk, None, None, None, None, None, None


def _prologue_grads(qkv, q_gamma, k_gamma, cos_t, sin_t, positions, rstd, dq, dk, dv, heads, head_dim, seq_len):
    """d(qkv) and the gamma gradients from dq, dk (rotated, normalised) and dv."""
    hk = heads * head_dim
    dqkv = torch.zeros_like(qkv) if dq is None or dk is None else torch.empty_like(qkv)
    dq = torch.zeros(qkv.shape[0], hk, device=qkv.device) if dq is None else dq.contiguous()
    dk = torch.zeros(qkv.shape[0], hk, device=qkv.device) if dk is None else dk.contiguous()
    dgq = torch.empty_like(q_gamma)
    dgk = torch.empty_like(k_gamma)
    ext().qk_prologue_bwd(qkv, q_gamma, k_gamma, cos_t, sin_t, positions, seq_len, dq, dk, rstd, dqkv, dgq, dgk,
                          heads, head_dim)
    if dv is None:
        dqkv[:, 2 * hk :] = 0.0
    else:
        dqkv[:, 2 * hk :].copy_(dv)
    return dqkv, dgq, dgk


class _QKVNormRope(torch.autograd.Function):
    """x -> (q, k, v) in one GEMM: the N-segmented QKV projection whose 3xTF32
    epilogue also RMS-normalises and rotates each q / k head of the row it
    holds, so the separate prologue pass over qkv disappears. The backward is
    the prologue backward followed by the projection's gradients."""

    @staticmethod
    def forward(ctx, x, wq, wk, wv, q_gamma, k_gamma, cos_t, sin_t, heads, head_dim, seq_len):
        x2 = x.reshape(-1, x.shape[-1])
        ws = [w.reshape(w.shape[0], -1) for w in (wq, wk, wv)]
        t, hk = x2.shape[0], heads * head_dim
        qkv = torch.empty(t, 3 * hk, device=x.device, dtype=torch.float32)
        q = torch.empty(t, hk, device=x.device, dtype=torch.float32)
        k = torch.empty_like(q)
        rstd = torch.empty(t * 2 * heads, device=x.device, dtype=torch.float32)
        ext().gemm_qkv_norm_rope(qkv, x2, ws, q, k, rstd, q_gamma, k_gamma, cos_t, sin_t, seq_len, heads, head_dim,
                                 EPS, precision.passes())
        ctx.save_for_backward(x2, wq, wk, wv, qkv, q_gamma, k_gamma, cos_t, sin_t, rstd)
        ctx.dims = (heads, head_dim, seq_len)
        ctx.x_shape = x.shape
        return q, k, qkv.narrow(1, 2 * hk, hk)

    @staticmethod
    def backward(ctx, dq, dk, dv):
        x2, wq, wk, wv, qkv, q_gamma, k_gamma, cos_t, sin_t, rstd = ctx.saved_tensors
        dqkv, dgq, dgk = _prologue_grads(qkv, q_gamma, k_gamma, cos_t, sin_t, None, rstd, dq, dk, dv, *ctx.dims)
        dx, dwq, dwk, dwv = gemm.qkv_projection_grads(x2, wq, wk, wv, dqkv)
        return dx.reshape(ctx.x_shape), dwq, dwk, dwv, dgq, dgk, None, None, None, None, None


class _Flash(torch.autograd.Function):
    """softmax(q k^T * scale, causal by position) v on tcgen05 tiles."""

    @staticmethod
    def forward(ctx, q, k, v, q_pos, k_pos, batch, heads, head_dim):
        lq = q.shape[0] // batch
        lk = k.shape[0] // batch
        out = torch.empty(q.shape[0], heads * head_dim, device=q.device, dtype=torch.float32)
        lse = torch.empty(batch, heads, lq, device=q.device, dtype=torch.float32)
        scale = 1.0 / math.sqrt(head_dim)
        ext().flash_attn_fwd(q, k, v, out, lse, batch, heads, head_dim, lq, lk, scale, q_pos, k_pos,
                             precision.passes())
        ctx.save_for_backward(q, k, v, out, lse, q_pos, k_pos)
        ctx.dims = (batch, heads, head_dim, lq, lk, scale)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out, lse, q_pos, k_pos = ctx.saved_tensors
        batch, heads, head_dim, lq, lk, scale = ctx.dims
        dq = torch.empty_like(q)
        dk = torch.empty(k.shape[0], heads * head_dim, device=k.device, dtype=torch.float32)
        dv = torch.empty_like(dk)
        ext().flash_attn_bwd(q, k, v, out, grad_out.contiguous(), lse, dq, dk, dv, batch, heads, head_dim, lq, lk,
                             scale, q_pos, k_pos, precision.passes())
        return dq, dk, dv, None, None, None, None, None


class _DenseCausal(torch.autograd.Function):
    """Materialised causal attention on the batched tcgen05 GEMM: S = scale QK^T
    (tiles above the diagonal skipped), in-place softmax, O = P V; backward
    dP = dO V^T, dS = P (dP - rowsum(P dP)) scale, dQ = dS K, dK = dS^T Q,
    dV = P^T dO. Used for head dims the fp32-accurate flash tiles do not cover
    (the reference's own formulation, ``abacus/attention.py:175-213``)."""

    @staticmethod
    def forward(ctx, q, k, v, batch, heads, head_dim):
        t = q.shape[0]
        length = t // batch
        scale = 1.0 / math.sqrt(head_dim)
        passes = precision.passes()

        def heads_view(x):
            return x.view(batch, length, heads, head_dim).permute(0, 2, 1, 3)

        s = torch.empty(batch, heads, length, length, device=q.device, dtype=torch.float32)
        ext().gemm_batched(s, heads_view(q), heads_view(k), False, True, scale, 1, passes)
        ext().causal_softmax_fwd(s)
        out = torch.empty(t, heads * head_dim, device=q.device, dtype=torch.float32)
        ext().gemm_batched(heads_view(out), s, heads_view(v), False, False, 1.0, 2, passes)
        ctx.save_for_backward(q, k, v, s)
        ctx.dims = (batch, heads, head_dim, length, scale)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, p = ctx.saved_tensors
        batch, heads, head_dim, length, scale = ctx.dims
        passes = precision.passes()

        def heads_view(x):
            return x.view(batch, length, heads, head_dim).permute(0, 2, 1, 3)

        do = heads_view(grad_out.contiguous())
        dp = torch.empty_like(p)
        ext().gemm_batched(dp, do, heads_view(v), False, True, 1.0, 1, passes)
        ext().causal_softmax_bwd(p, dp, scale)
        dq = torch.empty(q.shape[0], heads * head_dim, device=q.device, dtype=torch.float32)
        dk = torch.empty_like(dq)
        dv = torch.empty_like(dq)
        ext().gemm_batched(heads_view(dq), dp, heads_view(k), False, False, 1.0, 2, passes)
        ext().gemm_batched(heads_view(dk), dp, heads_view(q), True, False, 1.0, 3, passes)
        ext().gemm_batched(heads_view(dv), p, do, True, False, 1.0, 3, passes)
        return dq, dk, dv, None, None, None


def _flash_supports(head_dim: int) -> bool:
    """Head dims the flash kernels cover in the current precision mode."""
    if precision.passes() == 3:
        return head_dim in (32, 64)
    return head_dim in (32, 64, 128)


_TABLES: dict = {}


def _cached_tables(inv_freq: torch.Tensor, n_positions: int):
    key = (inv_freq.device, inv_freq.data_ptr(), n_positions, inv_freq._version)
    tables = _TABLES.get(key)
    if tables is None:
        if len(_TABLES) > 16:
            _TABLES.clear()
        tables = rope_tables(inv_freq, n_positions, inv_freq.device)
        _TABLES[key] = tables
    return tables


def qk_prologue(qkv, heads, head_dim, q_gamma, k_gamma, inv_freq, seq_len, positions=None, n_positions=None):
    """CUDA: RMSNorm q and k over head_dim, then RoPE (global ``positions``
    when given, else ``row % seq_len``). Returns (q, k, v) as (T, HK) tensors."""
    cos_t, sin_t = _cached_tables(inv_freq, n_positions or seq_len)
    return _QKPrologue.apply(qkv, q_gamma, k_gamma, cos_t, sin_t, positions, heads, head_dim, seq_len)


def flash_attention(q, k, v, batch, heads, head_dim, q_pos=None, k_pos=None):
    """CUDA flash attention over (T, HK) token-major tensors. Without positions
    the mask is plain causal over each sequence (requires Lq == Lk). Head dims
    without an fp32-accurate flash tile (128 in fp32 mode) take the
    materialised path for plain causal masks."""
    if not _flash_supports(head_dim):
        if q_pos is not None or k_pos is not None or q.shape[0] != k.shape[0]:
            raise NotImplementedError(
                f"head_dim {head_dim} in fp32 mode supports plain causal attention only (no positions)")
        return _DenseCausal.apply(q, k, v, batch, heads, head_dim)
    return _Flash.apply(q, k, v, q_pos, k_pos, batch, heads, head_dim)


def _fused_qk_usable(x: torch.Tensor, heads: int, head_dim: int, inv_freq) -> bool:
    return (x.is_cuda and inv_freq is not None and precision.passes() == 3 and head_dim in (64, 128)
            and (heads * head_dim) % 128 == 0 and os.environ.get("ABACUS_FUSED_QK", "1") != "0")


def qkv_attention(x, wq, wk, wv, batch, heads, head_dim, q_gamma, k_gamma, inv_freq):
    """x (..., D) -> (T, HK) attention output: QKV projection, QK-norm,
    RoPE and causal attention. On CUDA in fp32 mode the norm and rotation run
    in the projection GEMM's epilogue (``ABACUS_FUSED_QK=0``: separate
    prologue kernel); otherwise as ``causal_attention`` over the projection."""
    if _fused_qk_usable(x, heads, head_dim, inv_freq):
        seq_len = (x.numel() // x.shape[-1]) // batch
        cos_t, sin_t = _cached_tables(inv_freq, seq_len)
        q, k, v = _QKVNormRope.apply(x.contiguous(), wq, wk, wv, q_gamma.contiguous(), k_gamma.contiguous(), cos_t,
                                     sin_t, heads, head_dim, seq_len)
        return flash_attention(q, k, v, batch, heads, head_dim)
    qkv = gemm.qkv_projection(x, wq, wk, wv)
    return causal_attention(qkv, batch, heads, head_dim, q_gamma, k_gamma, inv_freq)


def causal_attention(
    qkv: torch.Tensor,
    batch: int,
    heads: int,
    head_dim: int,
    q_gamma: torch.Tensor,
    k_gamma: torch.Tensor,
    inv_freq: torch.Tensor | None,
) -> torch.Tensor:
    """(T, 3HK) projections -> (T, HK) attention output, causal over each row."""
    t = qkv.shape[0]
    seq_len = t // batch
    if not qkv.is_cuda or inv_freq is None:
        pos = torch.arange(seq_len, device=qkv.device)
        return attention_reference(qkv, batch, heads, head_dim, q_gamma, k_gamma, inv_freq, pos, pos)
    q, k, v = qk_prologue(qkv, heads, head_dim, q_gamma, k_gamma, inv_freq, seq_len)
    return flash_attention(q, k, v, batch, heads, head_dim)
