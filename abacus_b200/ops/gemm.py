"""GEMM entry points and the linear / SwiGLU autograd functions built on them.

Weights use the reference's (in, out) "math" layout (``x @ W``), e.g.
``abacus/mlp.py:23-25`` and ``abacus/attention.py:98-106``. On CUDA tensors
every product runs on the tcgen05 kernel in ``csrc/gemm`` (MN-major B for
``x @ W``, K-major B for ``dy @ W^T``, MN-major A and B for ``x^T @ dy``),
so no transposed copy of a weight or activation is ever made. On CPU tensors
the same math runs through ATen.
"""
from __future__ import annotations

import os

import torch

from abacus_b200.ops import precision
from abacus_b200.ops._ext import ext

B_SINGLE, B_SEG_N, B_SEG_K = 0, 1, 2


def _rows(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(-1, x.shape[-1])


def _transpose_for_wgrad() -> bool:
    # Off by default: on B200 the MN-major-A weight-gradient GEMM measured
    # faster (0.603 ms) than a transpose pass plus the K-major GEMM (0.622 ms)
    # on (32768 x 768)^T @ (32768 x 2048).
    return os.environ.get("ABACUS_WGRAD_TRANSPOSE", "0") == "1" and precision.passes() == 3


def transpose(a: torch.Tensor) -> torch.Tensor:
    """Contiguous (N, M) copy of a 2-D (M, N) fp32 CUDA tensor."""
    out = torch.empty(a.shape[1], a.shape[0], device=a.device, dtype=a.dtype)
    ext().transpose2d(a, out)
    return out


def matmul(
    a: torch.Tensor,
    b: torch.Tensor | list[torch.Tensor],
    *,
    trans_a: bool = False,
    trans_b: bool = False,
    b_mode: int = B_SINGLE,
    alpha: float = 1.0,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    accumulate: bool = False,
) -> torch.Tensor:
    """``out = alpha * op(a) @ op(b) [+ residual] [+ out]`` for 2-D fp32 tensors.

    ``op(a)`` is ``a`` (M, K) or ``a.T`` when ``trans_a`` (a stored (K, M)).
    ``op(b)`` is ``b`` (K, N) or ``b.T`` when ``trans_b`` (b stored (N, K)).
    A list of B tensors is concatenated along N (``B_SEG_N``) or K
    (``B_SEG_K``) without materialising the concatenation.
    """
    bs = list(b) if isinstance(b, (list, tuple)) else [b]
    if a.is_cuda:
        if trans_a and _transpose_for_wgrad():
            # Weight gradients x^T @ dy through a K-major copy of x (one HBM
            # pass), so the split converter reads A rows with 16-byte loads.
            a = transpose(a)
            trans_a = False
        m = a.shape[1] if trans_a else a.shape[0]
        if b_mode == B_SEG_N:
            n = sum((t.shape[0] if trans_b else t.shape[1]) for t in bs)
        else:
            n = bs[0].shape[0] if trans_b else bs[0].shape[1]
        if out is None:
            out = torch.empty(m, n, device=a.device, dtype=torch.float32)
            accumulate = False
        ext().gemm_out(out, a, bs, trans_a, trans_b, b_mode, float(alpha), residual, accumulate, precision.passes())
        return out
    # CPU formulation (oracle).
    lhs = a.t() if trans_a else a
    mats = [t.t() if trans_b else t for t in bs]
    if b_mode == B_SEG_N:
        rhs = torch.cat(mats, dim=1)
    elif b_mode == B_SEG_K:
        rhs = torch.cat(mats, dim=0)
    else:
        rhs = mats[0]
    result = alpha * (lhs @ rhs)
    if residual is not None:
        result = result + residual
    if out is not None:
        if accumulate:
            out.add_(result)
        else:
            out.copy_(result)
        return out
    return result


class _Linear(torch.autograd.Function):
    """``y = x @ W [+ residual]`` with W in (in, out) layout; the residual add
    is fused into the GEMM epilogue on the GPU."""

    @staticmethod
    def forward(ctx, x, weight, residual):
        x2 = _rows(x)
        res2 = None if residual is None else _rows(residual)
        y = matmul(x2, weight, residual=res2)
        ctx.save_for_backward(x2, weight)
        ctx.has_residual = residual is not None
        ctx.x_shape = x.shape
        return y.reshape(*x.shape[:-1], weight.shape[1])

    @staticmethod
    def backward(ctx, grad_y):
        x2, weight = ctx.saved_tensors
        g2 = _rows(grad_y).contiguous()
        grad_x = grad_w = None
        if ctx.needs_input_grad[0]:
            grad_x = matmul(g2, weight, trans_b=True).reshape(ctx.x_shape)
        if ctx.needs_input_grad[1]:
            grad_w = matmul(x2, g2, trans_a=True)
        grad_r = grad_y if ctx.has_residual and ctx.needs_input_grad[2] else None
        return grad_x, grad_w, grad_r


def linear(x: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
    if not x.is_cuda:
        y = x @ weight
        return y if residual is None else residual + y
    return _Linear.apply(x.contiguous(), weight, residual)


class _SwiGLU(torch.autograd.Function):
    """Fused SwiGLU MLP ``(silu(x @ Wg) * (x @ Wu)) @ Wd [+ residual]``.

    The gate/up GEMM writes gate, up and the product in one epilogue; the
    backward's first GEMM (``dy @ Wd^T``) applies the SwiGLU derivative in its
    epilogue, and ``dx`` is one K-segmented GEMM over ``[dgate | dup]``.
    Reference semantics: ``abacus/mlp.py:31-38``.
    """

    @staticmethod
    def forward(ctx, x, w_gate, w_up, w_down, residual):
        x2 = _rows(x)
        tokens, hidden = x2.shape[0], w_gate.shape[1]
        g = torch.empty(tokens, hidden, device=x.device, dtype=torch.float32)
        u = torch.empty_like(g)
        h = torch.empty_like(g)
        ext().gemm_swiglu(x2, w_gate, w_up, g, u, h, precision.passes())
        res2 = None if residual is None else _rows(residual)
        y = matmul(h, w_down, residual=res2)
        ctx.save_for_backward(x2, w_gate, w_up, w_down, g, u, h)
        ctx.has_residual = residual is not None
        ctx.x_shape = x.shape
        return y.reshape(*x.shape[:-1], w_down.shape[1])

    @staticmethod
    def backward(ctx, grad_y):
        x2, w_gate, w_up, w_down, g, u, h = ctx.saved_tensors
        g2 = _rows(grad_y).contiguous()
        hidden = w_gate.shape[1]
        dgu = torch.empty(g2.shape[0], 2 * hidden, device=g2.device, dtype=torch.float32)
        ext().gemm_swiglu_bwd(g2, w_down, g, u, dgu, precision.passes())
        if hidden % 32 == 0:
            grad_x = matmul(dgu, [w_gate, w_up], trans_b=True, b_mode=B_SEG_K)
        else:  # K segments must be whole 32-element k-tiles: two accumulating GEMMs
            grad_x = matmul(dgu[:, :hidden], w_gate, trans_b=True)
            matmul(dgu[:, hidden:], w_up, trans_b=True, out=grad_x, accumulate=True)
        grad_x = grad_x.reshape(ctx.x_shape)
        grad_wg = matmul(x2, dgu[:, :hidden], trans_a=True)
        grad_wu = matmul(x2, dgu[:, hidden:], trans_a=True)
        grad_wd = matmul(h, g2, trans_a=True)
        grad_r = grad_y if ctx.has_residual else None
        return grad_x, grad_wg, grad_wu, grad_wd, grad_r


def swiglu_mlp(
    x: torch.Tensor,
    w_gate: torch.Tensor,
    w_up: torch.Tensor,
    w_down: torch.Tensor,
    residual: torch.Tensor | None = None,
) -> torch.Tensor:
    if not x.is_cuda:
        y = (torch.nn.functional.silu(x @ w_gate) * (x @ w_up)) @ w_down
        return y if residual is None else residual + y
    return _SwiGLU.apply(x.contiguous(), w_gate, w_up, w_down, residual)


class _GroupedSwiGLU(torch.autograd.Function):
    """``_SwiGLU`` for E experts at once: x (E, C, D) holds every expert's C
    rows, w_gate / w_up (E, D, Mh), w_down (E, Mh, D). Each product is one
    grouped launch over all experts (``gemm_grouped`` / ``gemm_swiglu_grouped``),
    so the expert loop costs 2 forward and 6 backward launches for any E.
    """

    @staticmethod
    def forward(ctx, x, w_gate, w_up, w_down):
        n_exp, rows, _ = x.shape
        hidden = w_gate.shape[2]
        passes = precision.passes()
        g = torch.empty(n_exp, rows, hidden, device=x.device, dtype=torch.float32)
        u = torch.empty_like(g)
        h = torch.empty_like(g)
        ext().gemm_swiglu_grouped(x, w_gate, w_up, g, u, h, passes, None)
        y = torch.empty(n_exp, rows, w_down.shape[2], device=x.device, dtype=torch.float32)
        ext().gemm_grouped(y, h, [w_down], False, False, B_SINGLE, 1.0, False, passes, None)
        ctx.save_for_backward(x, w_gate, w_up, w_down, g, u, h)
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x, w_gate, w_up, w_down, g, u, h = ctx.saved_tensors
        gy = grad_y.contiguous()
        n_exp, rows, _ = x.shape
        hidden = w_gate.shape[2]
        passes = precision.passes()
        dgu = torch.empty(n_exp, rows, 2 * hidden, device=gy.device, dtype=torch.float32)
        ext().gemm_swiglu_bwd_grouped(gy, w_down, g, u, dgu, passes, None)
        dx = torch.empty_like(x)
        if hidden % 32 == 0:
            ext().gemm_grouped(dx, dgu, [w_gate, w_up], False, True, B_SEG_K, 1.0, False, passes, None)
        else:  # K segments must be whole 32-element k-tiles: two accumulating GEMMs
            ext().gemm_grouped(dx, dgu[..., :hidden], [w_gate], False, True, B_SINGLE, 1.0, False, passes, None)
            ext().gemm_grouped(dx, dgu[..., hidden:], [w_up], False, True, B_SINGLE, 1.0, True, passes, None)
        d_gate = torch.empty_like(w_gate)
        d_up = torch.empty_like(w_up)
        d_down = torch.empty_like(w_down)
        ext().gemm_grouped(d_gate, x, [dgu[..., :hidden]], True, False, B_SINGLE, 1.0, False, passes, None)
        ext().gemm_grouped(d_up, x, [dgu[..., hidden:]], True, False, B_SINGLE, 1.0, False, passes, None)
        ext().gemm_grouped(d_down, h, [gy], True, False, B_SINGLE, 1.0, False, passes, None)
        return dx, d_gate, d_up, d_down


def grouped_swiglu_mlp(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """Per-expert SwiGLU MLP over (E, C, D) rows: y[e] = (silu(x[e] Wg[e]) * (x[e] Wu[e])) Wd[e]."""
    if not x.is_cuda:
        return torch.bmm(torch.nn.functional.silu(torch.bmm(x, w_gate)) * torch.bmm(x, w_up), w_down)
    return _GroupedSwiGLU.apply(x.contiguous(), w_gate.contiguous(), w_up.contiguous(), w_down.contiguous())


class _QKVProjection(torch.autograd.Function):
    """``[x @ Wq | x @ Wk | x @ Wv]`` as one N-segmented GEMM (T, 3*HK).

    Weights stay three separate (D, H, K) parameters (the reference's layout,
    ``abacus/attention.py:98-111``); the kernel selects the B tensor per N
    tile, and the backward ``dx`` is one K-segmented GEMM over ``dqkv``.
    """

    @staticmethod
    def forward(ctx, x, wq, wk, wv):
        x2 = _rows(x)
        ws = [w.reshape(w.shape[0], -1) for w in (wq, wk, wv)]
        hk = ws[0].shape[1]
        if hk % 128 == 0:
            qkv = matmul(x2, ws, b_mode=B_SEG_N)
        else:
            qkv = torch.empty(x2.shape[0], 3 * hk, device=x.device, dtype=torch.float32)
            for i, w in enumerate(ws):
                matmul(x2, w, out=qkv[:, i * hk : (i + 1) * hk])
        ctx.save_for_backward(x2, wq, wk, wv)
        ctx.x_shape = x.shape
        return qkv

    @staticmethod
    def backward(ctx, dqkv):
        x2, wq, wk, wv = ctx.saved_tensors
        dx, *grads = qkv_projection_grads(x2, wq, wk, wv, dqkv)
        return (dx.reshape(ctx.x_shape), *grads)


def qkv_projection_grads(x2, wq, wk, wv, dqkv):
    """Gradients of ``[x @ Wq | x @ Wk | x @ Wv]`` given dqkv (T, 3*HK):
    dx (T, D) as one K-segmented GEMM, then dWq, dWk, dWv in their (D, H, K)
    shapes."""
    dqkv = dqkv.contiguous()
    ws = [w.reshape(w.shape[0], -1) for w in (wq, wk, wv)]
    hk = ws[0].shape[1]
    if hk % 32 == 0:
        dx = matmul(dqkv, ws, trans_b=True, b_mode=B_SEG_K)
    else:
        dx = matmul(dqkv[:, :hk].contiguous(), ws[0], trans_b=True)
        for i in (1, 2):
            matmul(dqkv[:, i * hk : (i + 1) * hk].contiguous(), ws[i], trans_b=True, out=dx, accumulate=True)
    grads = [matmul(x2, dqkv[:, i * hk : (i + 1) * hk], trans_a=True).view_as(w) for i, w in enumerate((wq, wk, wv))]
    return (dx, *grads)


def qkv_projection(x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor) -> torch.Tensor:
    """(..., D) -> (T, 3*H*K) with q | k | v column blocks."""
    if not x.is_cuda:
        x2 = x.reshape(-1, x.shape[-1])
        return torch.cat([x2 @ w.reshape(w.shape[0], -1) for w in (wq, wk, wv)], dim=1)
    return _QKVProjection.apply(x.contiguous(), wq, wk, wv)
