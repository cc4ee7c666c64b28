"""Trends over flushed observation history (flodl/src/graph/trend.rs):
least-squares slope, stalled / improving / converged predicates and groups."""
from __future__ import annotations

from typing import List, Sequence


def ols_slope(data: Sequence[float]) -> float:
    n = len(data)
    if n < 2:
        return 0.0
    sx = n * (n - 1) / 2.0
    sy = float(sum(data))
    sxy = float(sum(i * y for i, y in enumerate(data)))
    sxx = float(sum(i * i for i in range(n)))
    den = n * sxx - sx * sx
    if abs(den) < 1e-15:
        return 0.0
    return (n * sxy - sx * sy) / den


class Trend:
    def __init__(self, values: Sequence[float]):
        self._values = [float(v) for v in values]

    def __len__(self):
        return len(self._values)

    def is_empty(self) -> bool:
        return not self._values

    def values(self) -> List[float]:
        return list(self._values)

    def last(self, n: int) -> List[float]:
        return self._values[-n:] if n > 0 else list(self._values)

    def latest(self) -> float:
        return self._values[-1] if self._values else 0.0

    def mean(self) -> float:
        return sum(self._values) / len(self._values) if self._values else 0.0

    def min(self) -> float:
        return min(self._values) if self._values else 0.0

    def max(self) -> float:
        return max(self._values) if self._values else 0.0

    def slope(self, window: int = 0) -> float:
        return ols_slope(self.last(window))

    def stalled(self, window: int, tol: float) -> bool:
        return abs(self.slope(window)) < tol

    def improving(self, window: int) -> bool:
        return self.slope(window) < 0.0

    def converged(self, window: int, tol: float) -> bool:
        d = self.last(window)
        if len(d) < 2:
            return False
        m = sum(d) / len(d)
        return sum((v - m) ** 2 for v in d) / len(d) < tol


class TrendGroup:
    def __init__(self, trends: Sequence[Trend]):
        self.trends = list(trends)

    def __len__(self):
        return len(self.trends)

    def is_empty(self):
        return not self.trends

    def all_improving(self, window: int) -> bool:
        return bool(self.trends) and all(t.improving(window) for t in self.trends)

    def any_improving(self, window: int) -> bool:
        return any(t.improving(window) for t in self.trends)

    def all_stalled(self, window: int, tol: float) -> bool:
        return bool(self.trends) and all(t.stalled(window, tol) for t in self.trends)

    def any_stalled(self, window: int, tol: float) -> bool:
        return any(t.stalled(window, tol) for t in self.trends)

    def all_converged(self, window: int, tol: float) -> bool:
        return bool(self.trends) and all(t.converged(window, tol) for t in self.trends)

    def mean_slope(self, window: int) -> float:
        return sum(t.slope(window) for t in self.trends) / len(self.trends) if self.trends else 0.0
