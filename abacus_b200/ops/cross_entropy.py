"""Cross entropy with ``ignore_index`` (``F.cross_entropy`` semantics, as the
reference calls it at ``abacus/trainer.py:81-85`` and
``abacus/distributed/pipeline_parallel.py:56-61``), plus a fused
linear + cross-entropy that never materialises the full (T, V) logits.

``fused_linear_cross_entropy(h, W, targets)`` processes the tokens in chunks:
per chunk, one GEMM writes the logits, one kernel turns them in place into
``(softmax - onehot) * scale`` while producing the per-row loss, and two more
GEMMs accumulate ``dh = dlogits @ W^T`` and ``dW += h^T @ dlogits``. The
gradients are therefore ready when the forward returns; backward only scales
them by the incoming gradient. Peak extra memory is one (chunk, V) buffer.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from abacus_b200.ops import gemm
from abacus_b200.ops._ext import ext

IGNORE = -100


def _count(targets: torch.Tensor, ignore_index: int) -> torch.Tensor:
    return (targets != ignore_index).sum().to(torch.float32)


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, ignore_index, reduction):
        logits = logits.contiguous() if logits.stride(-1) != 1 or logits.stride(0) % 4 else logits
        target = target.contiguous()
        rows = logits.shape[0]
        loss = torch.empty(rows, device=logits.device, dtype=torch.float32)
        lse = torch.empty(rows, device=logits.device, dtype=torch.float32)
        one = torch.ones((), device=logits.device)
        ext().cross_entropy_fwd_bwd(logits, target, loss, lse, ignore_index, one, False)
        if reduction == "mean":
            denom = _count(target, ignore_index)
            out = loss.sum() / denom
        elif reduction == "sum":
            denom = one
            out = loss.sum()
        else:
            denom = None
            out = loss
        ctx.save_for_backward(logits, target, lse, denom if denom is not None else one)
        ctx.ignore_index = ignore_index
        ctx.reduction = reduction
        return out

    @staticmethod
    def backward(ctx, grad_out):
        logits, target, lse, denom = ctx.saved_tensors
        grad = torch.empty_like(logits)
        if ctx.reduction == "none":
            scale = torch.ones((), device=logits.device)
            ext().cross_entropy_grad(logits, grad, target, lse, ctx.ignore_index, scale)
            return grad * grad_out.unsqueeze(-1), None, None, None
        scale = (grad_out / denom).reshape(()).contiguous()
        ext().cross_entropy_grad(logits, grad, target, lse, ctx.ignore_index, scale)
        return grad, None, None, None


def cross_entropy(
    input: torch.Tensor,
    target: torch.Tensor,
    weight: torch.Tensor | None = None,
    size_average: bool | None = None,
    ignore_index: int = IGNORE,
    reduce: bool | None = None,
    reduction: str = "mean",
    label_smoothing: float = 0.0,
) -> torch.Tensor:
    """Drop-in for ``F.cross_entropy`` on 2-D logits. CUDA fp32 logits with the
    common arguments run on the abacus kernel; any other argument combination
    is rejected on CUDA rather than silently falling back."""
    if not input.is_cuda:
        return F.cross_entropy(
            input, target, weight=weight, size_average=size_average, ignore_index=ignore_index, reduce=reduce,
            reduction=reduction, label_smoothing=label_smoothing,
        )
    if weight is not None or size_average is not None or reduce is not None or label_smoothing != 0.0:
        raise NotImplementedError("abacus_b200 cross_entropy supports ignore_index and reduction only")
    if input.dim() != 2 or input.dtype != torch.float32:
        raise ValueError("cross_entropy expects (N, V) fp32 logits")
    return _CrossEntropy.apply(input, target, ignore_index, reduction)


class _FusedLinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, weight, targets, scale, chunk_rows):
        rows, dim = h.shape
        vocab = weight.shape[1]
        dh = torch.empty_like(h)
        dw = torch.zeros_like(weight)
        losses = torch.empty(rows, device=h.device, dtype=torch.float32)
        buf = torch.empty(min(chunk_rows, rows), vocab, device=h.device, dtype=torch.float32)
        for start in range(0, rows, chunk_rows):
            n = min(chunk_rows, rows - start)
            hc = h[start : start + n]
            logits = buf[:n]
            gemm.matmul(hc, weight, out=logits)
            ext().cross_entropy_fwd_bwd(logits, targets[start : start + n], losses[start : start + n], None, IGNORE,
                                        scale, True)
            gemm.matmul(logits, weight, trans_b=True, out=dh[start : start + n])
            gemm.matmul(hc, logits, trans_a=True, out=dw, accumulate=True)
        ctx.save_for_backward(dh, dw)
        return (losses.sum() * scale).reshape(())

    @staticmethod
    def backward(ctx, grad_out):
        dh, dw = ctx.saved_tensors
        return dh * grad_out, dw * grad_out, None, None, None


def fused_linear_cross_entropy(
    h: torch.Tensor,
    weight: torch.Tensor,
    targets: torch.Tensor,
    normalizer: torch.Tensor | float | None = None,
    chunk_rows: int = 8192,
) -> torch.Tensor:
    """``sum_i CE(h_i @ W, t_i) / normalizer`` over rows with ``t_i != -100``.

    ``h`` (T, D), ``weight`` (D, V) in the (in, out) layout, ``targets`` (T,).
    ``normalizer`` defaults to the number of non-ignored targets (the mean of
    ``F.cross_entropy``); pass a global count for token-weighted losses across
    ranks or microbatches.
    """
    h2 = h.reshape(-1, h.shape[-1])
    t2 = targets.reshape(-1)
    if normalizer is None:
        normalizer = _count(t2, IGNORE)
    if not h2.is_cuda:
        logits = h2 @ weight
        return F.cross_entropy(logits, t2, ignore_index=IGNORE, reduction="sum") / normalizer
    norm = torch.as_tensor(normalizer, device=h2.device, dtype=torch.float32).reshape(())
    scale = (1.0 / norm).contiguous()
    return _FusedLinearCE.apply(h2.contiguous(), weight, t2.contiguous(), scale, chunk_rows)
