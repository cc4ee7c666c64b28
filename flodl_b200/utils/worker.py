"""Background CPU jobs and a seedable random generator.

Reference roles: flodl/src/worker.rs (``CpuWorker``: fire-and-forget jobs
off the training thread - checkpoint writes, logging, metric export - with
``join`` to drain) and rng.rs (a small deterministic generator for
host-side shuffles and fixtures, independent of torch's global state).
"""
from __future__ import annotations

import queue
import threading
from typing import Callable, List, Optional


class CpuWorker:
    """One background thread executing submitted jobs in order. Errors are
    kept and re-raised by ``join``; the training thread never blocks on
    submission (unbounded queue)."""

    def __init__(self, name: str = "flodl-worker"):
        self.q: "queue.Queue[Optional[Callable[[], None]]]" = queue.Queue()
        self.errors: List[BaseException] = []
        self.done = 0
        self._t = threading.Thread(target=self._run, name=name, daemon=True)
        self._t.start()

    def _run(self):
        while True:
            job = self.q.get()
            if job is None:
                self.q.task_done()
                return
            try:
                job()
            except BaseException as e:  # surfaced by join()
                self.errors.append(e)
            finally:
                self.done += 1
                self.q.task_done()

    def submit(self, fn: Callable[[], None]) -> None:
        self.q.put(fn)

    def pending(self) -> int:
        return self.q.unfinished_tasks

    def join(self) -> None:
        """Wait for every submitted job; raise the first error if any failed."""
        self.q.join()
        if self.errors:
            e, self.errors = self.errors[0], []
            raise e

    def close(self) -> None:
        self.q.put(None)
        self._t.join(timeout=10)


class Rng:
    """SplitMix64 (Steele, Lea and Flood 2014): 64-bit state, one add and a
    mixing function per output; deterministic across platforms."""

    MASK = (1 << 64) - 1

    def __init__(self, seed: int = 0):
        self.state = seed & self.MASK

    def next_u64(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & self.MASK
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & self.MASK
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & self.MASK
        return z ^ (z >> 31)

    def uniform(self) -> float:
        return (self.next_u64() >> 11) * (1.0 / (1 << 53))

    def below(self, n: int) -> int:
        """Uniform integer in [0, n) by rejection (no modulo bias)."""
        if n <= 0:
            raise ValueError("n must be positive")
        limit = (1 << 64) - ((1 << 64) % n)
        while True:
            x = self.next_u64()
            if x < limit:
                return x % n

    def bernoulli(self, p: float) -> bool:
        return self.uniform() < p

    def shuffle(self, xs: list) -> list:
        """Fisher-Yates in place."""
        for i in range(len(xs) - 1, 0, -1):
            j = self.below(i + 1)
            xs[i], xs[j] = xs[j], xs[i]
        return xs
