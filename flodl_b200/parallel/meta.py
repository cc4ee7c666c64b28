"""LR-aware meta-controller above ElChe.

Reference: flodl/src/distributed/lr_event_meta.rs. Each averaging cycle it
records the learning rate, ElChe's anchor and the convergence guard's verdict
in short windows, and recommends shrinking the anchor
(``ElChe.nudge_anchor_down(factor)``) when

* the learning rate fell sharply in one cycle (``|dLR / LR_prev| > 0.3``:
  a step schedule's cliff; cosine decay stays below) - base factor 0.5; or
* the guard asked for a shrink (or suppressed growth) for the last ``K``
  cycles in a row - K and the base factor depend on ElChe's phase
  (warmup 5 / 0.3, stable 3 / 0.5, mature 2 / 0.7).

The factor is softened while ElChe is already shrinking the anchor and
strengthened while it grows (``base - (1 - base) x trend``, with trend =
(current anchor - window mean) / window mean), clamped to [0.1, 0.95]; when
both watchers fire the factors multiply. Nothing happens in the probe phase.
The window lengths, thresholds and factors are kept equal to the reference's
so cadence behaviour matches.
"""
from __future__ import annotations

import collections
from typing import Deque, Optional

PHASES = ("probe", "warmup", "stable", "mature")
_BASE = {"probe": 0.3, "warmup": 0.3, "stable": 0.5, "mature": 0.7}
_SUSTAIN = {"probe": 5, "warmup": 5, "stable": 3, "mature": 2}
LR_CLIFF_BASE = 0.5
SETTLED_EPS = 0.10


class LrEventMeta:
    def __init__(self, lr_window: int = 3, anchor_window: int = 5, guard_window: int = 5,
                 sharp_drop: float = 0.3, fmin: float = 0.1, fmax: float = 0.95):
        self.lrs: Deque[float] = collections.deque(maxlen=lr_window)
        self.anchors: Deque[int] = collections.deque(maxlen=anchor_window)
        self.verdicts: Deque[str] = collections.deque(maxlen=guard_window)
        self.sharp_drop, self.fmin, self.fmax = sharp_drop, fmin, fmax

    def anchor_trend(self) -> float:
        if len(self.anchors) < 2:
            return 0.0
        mean = sum(self.anchors) / len(self.anchors)
        return 0.0 if mean <= 0 else (self.anchors[-1] - mean) / mean

    def is_settled(self) -> bool:
        return abs(self.anchor_trend()) < SETTLED_EPS

    def _factor(self, base: float, trend: float) -> float:
        return min(max(base - (1.0 - base) * trend, self.fmin), self.fmax)

    def _cliff(self) -> bool:
        if len(self.lrs) < 2:
            return False
        prev, now = self.lrs[-2], self.lrs[-1]
        return prev > 0 and now < prev and (prev - now) / prev > self.sharp_drop

    def _sustained(self, phase: str) -> bool:
        k = _SUSTAIN[phase]
        if len(self.verdicts) < k:
            return False
        return all(v in ("shrink", "suppress_growth") for v in list(self.verdicts)[-k:])

    def observe(self, lr: float, anchor: int, verdict: str, phase: str) -> Optional[float]:
        """Record one cycle; the nudge factor to apply, or None."""
        self.lrs.append(float(lr))
        self.anchors.append(int(anchor))
        self.verdicts.append(verdict)
        if phase not in PHASES:
            raise ValueError(f"unknown phase {phase!r}")
        if phase == "probe":
            return None
        trend = self.anchor_trend()
        fs = []
        if self._cliff():
            fs.append(self._factor(LR_CLIFF_BASE, trend))
        if self._sustained(phase):
            fs.append(self._factor(_BASE[phase], trend))
        if not fs:
            return None
        f = fs[0] if len(fs) == 1 else min(max(fs[0] * fs[1], self.fmin), self.fmax)
        return f
