"""AdamW with the reference's exact update and ZeRO-slice support
(``abacus/optimizers/adamw.py``).

Per step and parameter: ``w *= 1 - lr*wd`` (every parameter, before the
moment update), ``m = lerp(m, g, 1-b1)``, ``v = b2 v + (1-b2) g^2``,
``w -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps)``. State is keyed by
``id(param)`` as ``{"step", "exp_avg", "exp_avg_sq"}``. With ``owned``
(ZeRO) only the owned flat slice of each parameter is stepped, using the
reduced shard in ``grad_shards`` when present.

On CUDA all parameters that share a step count are updated by one
multi-tensor kernel launch per 36 tensors (``csrc/ops/embed_ce_adamw.cu``);
on CPU the reference's per-parameter ATen sequence runs.
"""
from __future__ import annotations

import torch

from abacus_b200.ops._ext import ext


class AdamW:
    def __init__(
        self,
        model: torch.nn.Module,
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 1e-2,
        owned: dict[int, tuple[int, int]] | None = None,
        grad_shards: dict[int, torch.Tensor] | None = None,
    ):
        if lr < 0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if eps < 0:
            raise ValueError(f"Invalid epsilon: {eps}")
        if not 0.0 <= betas[0] < 1.0 or not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid betas: {betas}")
        if weight_decay < 0:
            raise ValueError(f"Invalid weight decay: {weight_decay}")
        self.params = list(model.parameters()) if isinstance(model, torch.nn.Module) else list(model)
        self.lr = lr
        self.beta1 = betas[0]
        self.beta2 = betas[1]
        self.eps = eps
        self.weight_decay = weight_decay
        self.owned = owned
        self.grad_shards = grad_shards
        self.state: dict[int, dict[str, torch.Tensor | int]] = {}
        if owned is not None:
            for param in self.params:
                bounds = owned.get(id(param))
                if bounds is None:
                    continue
                begin, end = bounds
                self.state[id(param)] = {
                    "step": 0,
                    "exp_avg": torch.zeros(end - begin, dtype=param.dtype, device=param.device),
                    "exp_avg_sq": torch.zeros(end - begin, dtype=param.dtype, device=param.device),
                }

    def zero_grad(self) -> None:
        for param in self.params:
            param.grad = None
        if self.grad_shards is not None:
            self.grad_shards.clear()

    def _weight_and_grad(self, param):
        if self.owned is None:
            return param, param.grad
        bounds = self.owned.get(id(param))
        if bounds is None:
            return param, None
        begin, end = bounds
        flat = param.data.reshape(-1)
        weight = flat if flat.numel() == end - begin else flat[begin:end]
        if self.grad_shards is not None and id(param) in self.grad_shards:
            return weight, self.grad_shards[id(param)]
        if param.grad is None:
            return weight, None
        grad = param.grad.reshape(-1)
        if grad.numel() != end - begin:
            grad = grad[begin:end]
        return weight, grad

    @torch.no_grad()
    def step(self) -> None:
        groups: dict[tuple, list] = {}
        for param in self.params:
            weight, grad = self._weight_and_grad(param)
            if grad is None:
                if self.owned is not None and id(param) in self.owned:
                    raise RuntimeError("sharded parameter is missing a gradient")
                continue
            if grad.is_sparse:
                raise RuntimeError("AdamW does not support sparse gradients")
            state = self.state.get(id(param))
            if state is None:
                state = {"step": 0, "exp_avg": torch.zeros_like(weight), "exp_avg_sq": torch.zeros_like(weight)}
                self.state[id(param)] = state
            state["step"] += 1
            if weight.is_cuda and weight.dtype == torch.float32:
                groups.setdefault((weight.device, state["step"]), []).append((weight, grad, state))
            else:
                self._step_reference(weight, grad, state)
        for (_, step), items in groups.items():
            weights = [w if w.is_contiguous() else w.contiguous() for w, _, _ in items]
            ext().adamw_step(
                weights,
                [g.contiguous() for _, g, _ in items],
                [s["exp_avg"] for _, _, s in items],
                [s["exp_avg_sq"] for _, _, s in items],
                float(self.lr), self.beta1, self.beta2, self.eps, self.weight_decay, int(step),
            )
            for (w, _, _), wc in zip(items, weights):
                if wc is not w:
                    w.copy_(wc)

    def _step_reference(self, weight, grad, state):
        exp_avg, exp_avg_sq = state["exp_avg"], state["exp_avg_sq"]
        if self.weight_decay != 0:
            weight.mul_(1 - self.lr * self.weight_decay)
        exp_avg.lerp_(grad, 1 - self.beta1)
        exp_avg_sq.mul_(self.beta2).addcmul_(grad, grad, value=1 - self.beta2)
        bias_correction1 = 1 - self.beta1 ** state["step"]
        bias_correction2 = 1 - self.beta2 ** state["step"]
        step_size = self.lr / bias_correction1
        denom = exp_avg_sq.sqrt().div_(bias_correction2**0.5).add_(self.eps)
        weight.addcdiv_(exp_avg, denom, value=-step_size)

    def state_dict_by_name(self, model: torch.nn.Module) -> dict:
        """Optimizer state keyed by parameter name (for checkpoints)."""
        out = {}
        for name, param in model.named_parameters():
            st = self.state.get(id(param))
            if st is not None:
                out[name] = {"step": st["step"], "exp_avg": st["exp_avg"], "exp_avg_sq": st["exp_avg_sq"]}
        return out

    def load_state_dict_by_name(self, model: torch.nn.Module, state: dict) -> None:
        for name, param in model.named_parameters():
            st = state.get(name)
            if st is None:
                continue
            self.state[id(param)] = {
                "step": int(st["step"]),
                "exp_avg": st["exp_avg"].to(device=param.device, dtype=param.dtype).clone(),
                "exp_avg_sq": st["exp_avg_sq"].to(device=param.device, dtype=param.dtype).clone(),
            }
