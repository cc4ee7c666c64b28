"""Convergence guards and weight-space divergence
(flodl/src/distributed/convergence.rs:163-520, divergence.rs:22).

divergence = ||pre - post|| / ||post|| of a rank's weights across an
averaging round. Guards turn the divergence history into a verdict on the
ElChe anchor: ``Stable`` (keep/grow), ``Shrink`` (nudge the anchor down).
"""
from __future__ import annotations

import enum
import math
from typing import List

import torch


def divergence(pre: torch.Tensor, post: torch.Tensor) -> float:
    num = torch.linalg.vector_norm((pre - post).float()).item()
    den = torch.linalg.vector_norm(post.float()).item()
    return num / den if den > 0 else 0.0


class Verdict(enum.Enum):
    STABLE = "stable"
    SHRINK = "shrink"


class ConvergenceGuard:
    def observe(self, div: float) -> Verdict:  # pragma: no cover - interface
        raise NotImplementedError


class NoGuard(ConvergenceGuard):
    def observe(self, div):
        return Verdict.STABLE


class LevelGuard(ConvergenceGuard):
    """Shrink when the divergence exceeds a fixed threshold."""

    def __init__(self, threshold: float = 0.05):
        self.threshold = threshold
        self.history: List[float] = []

    def observe(self, div):
        self.history.append(div)
        return Verdict.SHRINK if div > self.threshold else Verdict.STABLE


class GrowthGuard(ConvergenceGuard):
    """Shrink when divergence grows for ``patience`` consecutive rounds."""

    def __init__(self, patience: int = 3, rel: float = 0.05):
        self.patience, self.rel = patience, rel
        self.history: List[float] = []
        self._streak = 0

    def observe(self, div):
        if self.history and div > self.history[-1] * (1 + self.rel):
            self._streak += 1
        else:
            self._streak = 0
        self.history.append(div)
        return Verdict.SHRINK if self._streak >= self.patience else Verdict.STABLE


def realized_mass(batches: int, gamma: float) -> float:
    """Work mass of a rank for the weighted average: n^gamma
    (flodl/src/distributed/realized_work.rs:54-78)."""
    return float(batches) ** gamma if batches > 0 else 0.0
