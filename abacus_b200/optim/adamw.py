"""AdamW (``abacus/optimizers/adamw.py``) with ZeRO-slice support.

Update of one step (t = the parameter's own step count, lr / betas / eps / wd
the optimizer's):

    w  <- w * (1 - lr * wd)                  every parameter, before the moments
    m  <- lerp(m, g, 1 - b1)
    v  <- b2 * v + (1 - b2) * g * g
    w  <- w - lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)

The interface is the reference's: the constructor takes the model, ``owned``
maps ``id(param)`` to the flat range ``[begin, end)`` this rank updates under
ZeRO (moments are allocated for exactly that range up front), ``grad_shards``
holds the already-reduced gradient of that range (ZeRO-2/3), and the state of
a parameter is ``{"step", "exp_avg", "exp_avg_sq"}`` keyed by ``id(param)``.

Execution: parameters are grouped by (device, step count). On CUDA each group
is one multi-tensor kernel launch per 36 tensors (``csrc/ops/embed_ce_adamw.cu``);
elsewhere each group runs the same update as ``torch._foreach_*`` operations,
which apply the formulas above element by element in the order written.
"""
from __future__ import annotations

import torch

from abacus_b200.ops._ext import ext

_NOT_OWNED = object()


def _check_hyperparameters(lr: float, betas: tuple[float, float], eps: float, weight_decay: float) -> None:
    problems = []
    if not lr >= 0:
        problems.append(f"lr={lr!r} (must be >= 0)")
    if not eps >= 0:
        problems.append(f"eps={eps!r} (must be >= 0)")
    if len(betas) != 2 or not all(0.0 <= b < 1.0 for b in betas):
        problems.append(f"betas={tuple(betas)!r} (each must be in [0, 1))")
    if not weight_decay >= 0:
        problems.append(f"weight_decay={weight_decay!r} (must be >= 0)")
    if problems:
        raise ValueError("AdamW: invalid " + ", ".join(problems))


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
        _check_hyperparameters(lr, betas, eps, weight_decay)
        self.params = list(model.parameters()) if isinstance(model, torch.nn.Module) else list(model)
        self.lr = lr
        self.beta1, self.beta2 = float(betas[0]), float(betas[1])
        self.eps = eps
        self.weight_decay = weight_decay
        self.owned = owned
        self.grad_shards = grad_shards
        self.state: dict[int, dict[str, torch.Tensor | int]] = {}
        for param in self.params if owned is not None else ():
            span = owned.get(id(param))
            if span is not None:
                self.state[id(param)] = self._fresh_state(span[1] - span[0], param)

    @staticmethod
    def _fresh_state(numel: int, like: torch.Tensor) -> dict:
        zeros = lambda: torch.zeros(numel, dtype=like.dtype, device=like.device)  # noqa: E731
        return {"step": 0, "exp_avg": zeros(), "exp_avg_sq": zeros()}

    def zero_grad(self) -> None:
        for param in self.params:
            param.grad = None
        if self.grad_shards:
            self.grad_shards.clear()

    # ------------------------------------------------------------ selection
    def _span(self, param):
        """Flat range this rank updates: None = the whole tensor (no ZeRO),
        ``_NOT_OWNED`` = nothing, else ``(begin, end)``."""
        if self.owned is None:
            return None
        return self.owned.get(id(param), _NOT_OWNED)

    def _operands(self, param, span):
        """(weight, grad) tensors that this step updates / reads for ``param``.

        Under ZeRO the weight is the owned range of the flattened parameter
        (stage 3 stores only that range, so it is the whole storage). The
        gradient is the reduced shard if one was handed over, else the same
        range of ``param.grad`` (stage 1), else None.
        """
        if span is None:
            return param, param.grad
        lo, hi = span
        flat_w = param.data.view(-1)
        weight = flat_w[lo:hi] if flat_w.numel() != hi - lo else flat_w
        reduced = self.grad_shards.get(id(param)) if self.grad_shards is not None else None
        if reduced is not None:
            return weight, reduced
        if param.grad is None:
            return weight, None
        flat_g = param.grad.reshape(-1)
        return weight, (flat_g[lo:hi] if flat_g.numel() != hi - lo else flat_g)

    # ------------------------------------------------------------ update
    @torch.no_grad()
    def step(self) -> None:
        groups: dict[tuple, list] = {}
        for param in self.params:
            span = self._span(param)
            if span is _NOT_OWNED:
                continue
            weight, grad = self._operands(param, span)
            if grad is None:
                if span is not None:
                    # Stepping the other owned parameters without this one
                    # would put the ranks' step counts out of line.
                    raise RuntimeError(f"AdamW: owned ZeRO slice of a {tuple(param.shape)} parameter is missing a gradient")
                continue
            if grad.is_sparse:
                raise RuntimeError("AdamW: sparse gradients are not supported")
            state = self.state.get(id(param))
            if state is None:
                state = self.state[id(param)] = self._fresh_state(weight.numel(), weight)
            if state["exp_avg"].shape != weight.shape:  # flat moments of a whole parameter
                state["exp_avg"] = state["exp_avg"].view(weight.shape)
                state["exp_avg_sq"] = state["exp_avg_sq"].view(weight.shape)
            state["step"] += 1
            key = (weight.device, state["step"], weight.is_cuda and weight.dtype == torch.float32)
            groups.setdefault(key, []).append((weight, grad, state))
        for (_, step, on_kernel), items in groups.items():
            (self._launch_kernel if on_kernel else self._foreach_update)(items, step)

    def _launch_kernel(self, items, step: int) -> None:
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

    def _foreach_update(self, items, step: int) -> None:
        weights = [w for w, _, _ in items]
        grads = [g.to(w.dtype) if g.dtype != w.dtype else g for w, g, _ in items]
        m = [s["exp_avg"] for _, _, s in items]
        v = [s["exp_avg_sq"] for _, _, s in items]
        if self.weight_decay != 0:
            torch._foreach_mul_(weights, 1 - self.lr * self.weight_decay)
        torch._foreach_lerp_(m, grads, 1 - self.beta1)
        torch._foreach_mul_(v, self.beta2)
        torch._foreach_addcmul_(v, grads, grads, value=1 - self.beta2)
        correction1 = 1 - self.beta1 ** step
        correction2 = 1 - self.beta2 ** step
        denom = torch._foreach_sqrt(v)
        torch._foreach_div_(denom, correction2 ** 0.5)
        torch._foreach_add_(denom, self.eps)
        torch._foreach_addcdiv_(weights, m, denom, value=-(self.lr / correction1))

    # ------------------------------------------------------------ checkpoints
    def state_dict_by_name(self, model: torch.nn.Module) -> dict:
        """Optimizer state keyed by parameter name (for checkpoints)."""
        named = ((name, self.state.get(id(p))) for name, p in model.named_parameters())
        return {name: {k: st[k] for k in ("step", "exp_avg", "exp_avg_sq")} for name, st in named if st is not None}

    def load_state_dict_by_name(self, model: torch.nn.Module, state: dict) -> None:
        for name, param in model.named_parameters():
            saved = state.get(name)
            if saved is None:
                continue
            self.state[id(param)] = {
                "step": int(saved["step"]),
                "exp_avg": saved["exp_avg"].to(device=param.device, dtype=param.dtype).clone(),
                "exp_avg_sq": saved["exp_avg_sq"].to(device=param.device, dtype=param.dtype).clone(),
            }
