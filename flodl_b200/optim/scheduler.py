"""Learning-rate schedules (flodl/src/nn/scheduler.rs). Each maps a step index
to a learning rate; ``WarmupScheduler`` composes with any inner schedule."""
from __future__ import annotations

import math
from typing import Sequence


class Scheduler:
    def lr(self, step: int) -> float:  # pragma: no cover - interface
        raise NotImplementedError

    def __call__(self, step: int) -> float:
        return self.lr(step)


class StepDecay(Scheduler):
    def __init__(self, base_lr: float, step_size: int, gamma: float):
        if step_size < 1:
            raise ValueError(f"StepDecay: step_size must be >= 1, got {step_size}")
        self.base_lr, self.step_size, self.gamma = base_lr, step_size, gamma

    def lr(self, step):
        return self.base_lr * self.gamma ** (step // self.step_size)


class CosineScheduler(Scheduler):
    def __init__(self, base_lr: float, min_lr: float, total_steps: int):
        if total_steps < 1:
            raise ValueError(f"CosineScheduler: total_steps must be >= 1, got {total_steps}")
        self.base_lr, self.min_lr, self.total_steps = base_lr, min_lr, total_steps

    def lr(self, step):
        t = min(step, self.total_steps) / self.total_steps
        return self.min_lr + 0.5 * (self.base_lr - self.min_lr) * (1 + math.cos(math.pi * t))


class WarmupScheduler(Scheduler):
    """Linear warmup to ``target_lr`` over ``warmup_steps``, then ``inner``
    (indexed from the end of warmup)."""

    def __init__(self, inner: Scheduler, target_lr: float, warmup_steps: int):
        self.inner, self.target_lr, self.warmup_steps = inner, target_lr, warmup_steps

    def lr(self, step):
        if step < self.warmup_steps:
            return self.target_lr * (step + 1) / self.warmup_steps
        return self.inner.lr(step - self.warmup_steps)


class PlateauScheduler:
    """Reduce the lr by ``factor`` after ``patience`` non-improving observations."""

    def __init__(self, base_lr: float, patience: int, factor: float, min_lr: float):
        self.patience, self.factor, self.min_lr = patience, factor, min_lr
        self.current_lr = base_lr
        self.best = math.inf
        self.wait = 0

    def observe(self, metric: float) -> float:
        if metric < self.best:
            self.best = metric
            self.wait = 0
        else:
            self.wait += 1
            if self.wait >= self.patience:
                self.current_lr = max(self.current_lr * self.factor, self.min_lr)
                self.wait = 0
        return self.current_lr

    def lr(self, step: int = 0) -> float:
        return self.current_lr


class ExponentialLR(Scheduler):
    def __init__(self, base_lr: float, gamma: float):
        self.base_lr, self.gamma = base_lr, gamma

    def lr(self, step):
        return self.base_lr * self.gamma ** step


class MultiStepLR(Scheduler):
    def __init__(self, base_lr: float, milestones: Sequence[int], gamma: float):
        self.base_lr, self.milestones, self.gamma = base_lr, sorted(milestones), gamma

    def lr(self, step):
        n = sum(1 for m in self.milestones if step >= m)
        return self.base_lr * self.gamma ** n


class OneCycleLR(Scheduler):
    """Linear warmup from max_lr/25 to max_lr, then cosine anneal back."""

    def __init__(self, max_lr: float, total_steps: int, warmup_frac: float = 0.3):
        self.max_lr, self.total_steps = max_lr, total_steps
        self.warmup_steps = int(round(total_steps * min(max(warmup_frac, 0.0), 1.0)))

    @classmethod
    def with_warmup_frac(cls, max_lr, total_steps, warmup_frac):
        return cls(max_lr, total_steps, warmup_frac)

    def lr(self, step):
        step = min(step, self.total_steps)
        lo = self.max_lr / 25.0
        if step < self.warmup_steps:
            return lo + step / max(self.warmup_steps, 1) * (self.max_lr - lo)
        decay = max(self.total_steps - self.warmup_steps, 1)
        t = (step - self.warmup_steps) / decay
        return lo + 0.5 * (self.max_lr - lo) * (1 + math.cos(math.pi * t))


class CyclicLR(Scheduler):
    def __init__(self, base_lr: float, max_lr: float, step_size: int, step_size_down: int = None):
        if step_size < 1 or (step_size_down is not None and step_size_down < 1):
            raise ValueError("CyclicLR: step sizes must be >= 1")
        self.base_lr, self.max_lr = base_lr, max_lr
        self.up = step_size
        self.down = step_size_down if step_size_down is not None else step_size

    @classmethod
    def asymmetric(cls, base_lr, max_lr, up, down):
        return cls(base_lr, max_lr, up, down)

    def lr(self, step):
        pos = step % (self.up + self.down)
        scale = pos / self.up if pos <= self.up else 1.0 - (pos - self.up) / self.down
        return self.base_lr + (self.max_lr - self.base_lr) * scale
