"""Outer optimizers applied to the cluster consensus (flodl/src/distributed/
outer_optimizer.rs:70-330), operating on flat parameter vectors.

Pseudo-gradient g = prev_global - consensus.
* ``OuterAvg``:          new = consensus (plain averaging)
* ``SlowMomentum``:      v = mu v + g;            new = prev - lr v   (SlowMo, Wang et al. 2019)
* ``NesterovMomentum``:  v = mu v + g;            new = prev - lr (mu v + g)
                          and the inner optimizer state is reset (DiLoCo, Douillard et al. 2023)
"""
from __future__ import annotations

from typing import Optional

import torch


class OuterOptimizer:
    resets_inner = False

    def outer_step(self, prev_global: torch.Tensor, consensus: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def state(self) -> Optional[torch.Tensor]:
        return None

    def load_state(self, t: torch.Tensor) -> None:
        pass


class OuterAvg(OuterOptimizer):
    def outer_step(self, prev_global, consensus):
        return consensus


class SlowMomentum(OuterOptimizer):
    def __init__(self, lr: float = 1.0, mu: float = 0.5):
        self.lr, self.mu = lr, mu
        self.v: Optional[torch.Tensor] = None

    def outer_step(self, prev_global, consensus):
        g = prev_global - consensus
        self.v = g if self.v is None or self.v.shape != g.shape else self.v * self.mu + g
        return prev_global - self.lr * self.v

    def state(self):
        return self.v

    def load_state(self, t):
        self.v = t


class NesterovMomentum(SlowMomentum):
    resets_inner = True

    def __init__(self, lr: float = 0.7, mu: float = 0.9):
        super().__init__(lr, mu)

    def outer_step(self, prev_global, consensus):
        g = prev_global - consensus
        self.v = g.clone() if self.v is None or self.v.shape != g.shape else self.v * self.mu + g
        return prev_global - self.lr * (self.v * self.mu + g)


class OuterStepper:
    """Holds the previous global model and applies an OuterOptimizer to each
    consensus (controller side)."""

    def __init__(self, opt: OuterOptimizer):
        self.opt = opt
        self.prev: Optional[torch.Tensor] = None

    def step(self, consensus: torch.Tensor) -> torch.Tensor:
        if self.prev is None:
            self.prev = consensus.clone()
            return consensus
        new = self.opt.outer_step(self.prev, consensus)
        self.prev = new.clone()
        return new


def easgd_blend(local: torch.Tensor, center: torch.Tensor, alpha: float) -> torch.Tensor:
    """Elastic averaging: local <- (1 - alpha) local + alpha center."""
    return local.mul_(1.0 - alpha).add_(center, alpha=alpha)
