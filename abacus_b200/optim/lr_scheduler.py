"""Warmup-stable-decay learning-rate schedule (``abacus/optimizers/lr_scheduler.py``).

The schedule is a piecewise-linear function of the 1-based step ``s`` in
``[1, T]`` with peak ``lr``:

    ramp   s in [1, W]          lr * s / W             (W = floor(0.02 T))
    hold   s in (W, T - D]      lr
    decay  s in (T - D, T]      lr * (1 - (s - (T - D)) / D)   (D = floor(0.10 T))

W + D <= 0.12 T, so the ramp and the decay never overlap; a zero-length phase
is skipped. The arithmetic of each phase is the reference's, so both produce
the same floating-point values.
"""
from __future__ import annotations

_WARMUP_PERCENT = 2
_DECAY_PERCENT = 10


class WSD:
    def __init__(self, total_steps: int, lr: float = 5e-4):
        if not (isinstance(total_steps, int) and total_steps >= 1):
            raise ValueError(f"WSD needs total_steps >= 1 (got {total_steps!r})")
        if not lr >= 0:
            raise ValueError(f"WSD needs a non-negative peak learning rate (got {lr!r})")
        self.total_steps = total_steps
        self.lr = lr
        self.warmup_steps = total_steps * _WARMUP_PERCENT // 100
        self.decay_steps = total_steps * _DECAY_PERCENT // 100
        self._decay_start = total_steps - self.decay_steps  # last step of the hold phase
        self._step = 0

    def learning_rate(self, step: int) -> float:
        """Learning rate of 1-based step ``step``."""
        if not 1 <= step <= self.total_steps:
            raise ValueError(f"WSD step {step} is outside the schedule's 1..{self.total_steps}")
        if step <= self.warmup_steps:  # empty when warmup_steps == 0
            return self.lr * step / self.warmup_steps
        if step > self._decay_start:  # empty when decay_steps == 0
            return self.lr * (1 - (step - self._decay_start) / self.decay_steps)
        return self.lr

    def step(self) -> float:
        """Advance one step and return its learning rate."""
        self._step += 1
        return self.learning_rate(self._step)

    def state_dict(self) -> dict:
        return {"total_steps": self.total_steps, "lr": self.lr, "step": self._step}

    def load_state_dict(self, state: dict) -> None:
        self._step = int(state["step"])
