"""Convergence guards and weight-space divergence
(flodl/src/distributed/convergence.rs:163-520, divergence.rs:22).

divergence = ||pre - post|| / ||post|| of a rank's weights across an
averaging round. Guards turn the divergence history into a verdict on the
ElChe anchor: ``Stable`` (commit growth), ``Suppress`` (veto growth) or
``Nudge`` (shrink the anchor).
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
    """A guard's verdict on the ElChe anchor (the reference's
    ``ConvergenceAction``): ``STABLE`` commits a pending window-growth
    proposal, ``SUPPRESS`` vetoes it and latches growth off, ``NUDGE``
    discards it and scales the anchor down by the guard's factor."""
    STABLE = "stable"
    SUPPRESS = "suppress"
    NUDGE = "nudge"
    SHRINK = "nudge"  # older name of NUDGE


class ConvergenceGuard:
    nudge_factor = 0.5

    def observe(self, div: float) -> Verdict:  # pragma: no cover - interface
        raise NotImplementedError

    def trend_history(self) -> List[float]:
        return list(getattr(self, "history", []))

    def reset(self) -> None:
        if hasattr(self, "history"):
            self.history.clear()


class NoGuard(ConvergenceGuard):
    def observe(self, div):
        return Verdict.STABLE


class LevelGuard(ConvergenceGuard):
    """Production default: the last five divergences are kept; three strictly
    rising readings whose latest is above ``threshold`` suppress growth.
    (flodl/src/distributed/ddp_run/convergence.rs:361-470)"""

    def __init__(self, threshold: float = 0.05, history=None):
        self.threshold = threshold
        self.history: List[float] = list(history or [])[-5:]

    def observe(self, div):
        self.history.append(float(div))
        del self.history[:-5]
        h = self.history
        if len(h) >= 3 and h[-1] > h[-2] > h[-3] and h[-1] > self.threshold:
            return Verdict.SUPPRESS
        return Verdict.STABLE


class GrowthGuard(ConvergenceGuard):
    """Divergence-growth guard: a reading more than ``rel`` above the previous
    one extends a rising streak; ``suppress_sustain`` rising readings
    suppress growth, ``nudge_sustain`` rising readings above
    ``nudge_threshold`` nudge the anchor down by ``nudge_factor``."""

    def __init__(self, rel: float = 0.05, suppress_sustain: int = 3, nudge_sustain: int = 3,
                 nudge_threshold: float = 1e-2, nudge_factor: float = 0.5, patience=None):
        if patience is not None:
            suppress_sustain = nudge_sustain = patience
        self.rel = rel
        self.suppress_sustain, self.nudge_sustain = suppress_sustain, nudge_sustain
        self.nudge_threshold, self.nudge_factor = nudge_threshold, nudge_factor
        self.history: List[float] = []
        self._streak = 0

    def observe(self, div):
        if self.history and div > self.history[-1] * (1 + self.rel):
            self._streak += 1
        else:
            self._streak = 0
        self.history.append(float(div))
        del self.history[:-64]
        if self._streak >= self.nudge_sustain and div > self.nudge_threshold:
            self._streak = 0
            return Verdict.NUDGE
        if self._streak >= self.suppress_sustain:
            return Verdict.SUPPRESS
        return Verdict.STABLE


def realized_mass(batches: int, gamma: float) -> float:
    """Work mass of a rank for the weighted average: n^gamma
    (flodl/src/distributed/realized_work.rs:54-78)."""
    return float(batches) ** gamma if batches > 0 else 0.0
