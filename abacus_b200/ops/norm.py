"""RMSNorm ``gamma * x / sqrt(mean(x^2) + eps)`` (``abacus/norm.py:23-31``).

CUDA: one fused forward kernel (saves 1/rms per row) and one backward kernel
that produces dx and per-block dgamma partials reduced by a second pass.
"""
from __future__ import annotations

import torch

from abacus_b200.ops._ext import ext

EPS = 1e-5


def rmsnorm_reference(x: torch.Tensor, gamma: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    rms = torch.sqrt(x.square().mean(dim=-1, keepdim=True) + eps)
    return gamma * x / rms


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, eps):
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], device=x.device, dtype=torch.float32)
        ext().rmsnorm_fwd(x2, gamma, y, rstd, float(eps))
        ctx.save_for_backward(x2, gamma, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, grad_y):
        x2, gamma, rstd = ctx.saved_tensors
        g2 = grad_y.reshape(-1, grad_y.shape[-1]).contiguous()
        dx = torch.empty_like(x2)
        dgamma = torch.empty_like(gamma)
        ext().rmsnorm_bwd(g2, x2, gamma, rstd, dx, dgamma)
        return dx.view(ctx.shape), dgamma, None


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    if not x.is_cuda:
        return rmsnorm_reference(x, gamma, eps)
    return _RMSNorm.apply(x, gamma, eps)
