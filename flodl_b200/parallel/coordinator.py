"""Cluster coordinator pieces: progressive epoch dispatch, window ledger,
callback-role election and the alert lane.

Reference roles: flodl/src/distributed/chunk_pool.rs (spans, cursors,
stealing, forfeit, coverage - native, csrc/runtime/chunk_pool.cpp),
cluster_coordinator/window_ledger.rs, callback_roles.rs and alerts.rs.

Progressive dispatch: an epoch's permutation (offsets ``0..total``) is split
into contiguous per-rank spans sized by measured throughput. A rank's chunks
come from the front of its own span, so its upcoming data is deterministic
(stageable ahead). A rank that exhausts its span steals from the tail of the
largest remaining span - owner front-to-back, thief back-to-front, so they
never overlap. Chunks of a dead rank that were dispatched but not completed
are forfeited back to the pool and re-dispatched first. ``uncovered_ranges``
(everything not dispatched-and-completed) is what a checkpoint records;
``ChunkPool.from_coverage`` resumes with exactly those holes.
"""
from __future__ import annotations

import collections
import time
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Sequence, Tuple


def spans_from_throughput(total: int, rates: Sequence[float]) -> List[int]:
    """Split ``total`` samples proportionally to per-rank rates (equal when
    uncalibrated); the last rank absorbs rounding."""
    n = len(rates)
    if n == 0:
        return []
    if not all(r > 0 for r in rates):
        rates = [1.0] * n
    s = sum(rates)
    out = [int(total * r / s) for r in rates[:-1]]
    out.append(total - sum(out))
    return out


class ChunkPool:
    """Progressive dispatch pool. The state machine lives in the native
    runtime (``flodl_b200._native.ChunkPool``); constructing this class
    returns that object, whose methods are ``take_chunk(size, rank)``,
    ``rollback_take``, ``mark_completed``, ``forfeit``, ``residue``,
    ``reservation``, ``remaining``, ``in_flight``, ``is_epoch_done``,
    ``uncovered_ranges`` and the ``completed`` counter."""

    def __new__(cls, epoch: int, total: int, spans: Sequence[int]):
        from .._ext import native
        return native().ChunkPool(int(epoch), int(total), [int(s) for s in spans])

    @staticmethod
    def equal(epoch: int, total: int, world: int):
        return ChunkPool(epoch, total, spans_from_throughput(total, [1.0] * world))

    @staticmethod
    def from_coverage(epoch: int, total: int, world: int, uncovered: Sequence[Tuple[int, int]]):
        """A pool whose only work is the ``uncovered`` (offset, size) ranges."""
        from .._ext import native
        return native().ChunkPool.from_coverage(int(epoch), int(total), int(world),
                                                [(int(o), int(n)) for o, n in uncovered])


# ----------------------------------------------------------------- window ledger
@dataclass
class _RankWindow:
    batches: int = 0
    samples: int = 0
    wall_ms: float = 0.0
    first_ms: Optional[float] = None
    excluded_ms: float = 0.0


class WindowLedger:
    """Per-rank bookkeeping of the current averaging window (advisory
    scheduling state; the reduce's divisor is the mass the ranks report)."""

    def __init__(self, world: int):
        self.w = [_RankWindow() for _ in range(world)]

    def record_batch(self, rank: int, samples: int, wall_ms: float) -> None:
        r = self.w[rank]
        if r.first_ms is None:
            r.first_ms = wall_ms  # carries the window's fill (plan pickup, prefetch spin-up)
        r.batches += 1
        r.samples += samples
        r.wall_ms += wall_ms

    def exclude(self, rank: int, ms: float) -> None:
        """Wall time spent in callbacks (eval, checkpoint) that is not training."""
        self.w[rank].excluded_ms += ms

    def per_batch_ms(self, rank: int) -> Optional[float]:
        """Marginal per-batch wall time: the first batch (with the fill) excluded."""
        r = self.w[rank]
        if r.batches < 2:
            return r.first_ms
        return max(0.0, r.wall_ms - r.first_ms - r.excluded_ms) / (r.batches - 1)

    def fill_excess_ms(self, rank: int) -> float:
        r = self.w[rank]
        m = self.per_batch_ms(rank)
        return max(0.0, (r.first_ms or 0.0) - (m or 0.0))

    def delivered_rate(self, rank: int) -> Optional[float]:
        """Samples per ms at the marginal rate."""
        m = self.per_batch_ms(rank)
        r = self.w[rank]
        if not m or not r.batches:
            return None
        return (r.samples / r.batches) / m

    def batches(self, rank: int) -> int:
        return self.w[rank].batches

    def reset(self) -> None:
        self.w = [_RankWindow() for _ in self.w]


# ----------------------------------------------------------------- callback roles
class CallbackRoles:
    """Sticky election of the rank that runs epoch/eval/checkpoint callbacks:
    the fastest alive rank, replaced only when another is faster by
    ``margin`` (hysteresis) or the holder dies."""

    def __init__(self, world: int, margin: float = 0.10):
        self.alive = set(range(world))
        self.margin = margin
        self.holder = 0

    def observe(self, per_batch_ms: Dict[int, float]) -> int:
        cand = {r: m for r, m in per_batch_ms.items() if r in self.alive and m and m > 0}
        if not cand:
            return self.holder
        best = min(cand, key=cand.get)
        cur = cand.get(self.holder)
        if self.holder not in self.alive or cur is None or cand[best] < cur * (1 - self.margin):
            self.holder = best
        return self.holder

    def rank_died(self, rank: int) -> int:
        self.alive.discard(rank)
        if self.holder == rank and self.alive:
            self.holder = min(self.alive)  # failover; re-elected on the next observation
        return self.holder


# ----------------------------------------------------------------- alert lane
ALERT_CLASSES = ("rank_lost", "drift", "control_drop")


class AlertLane:
    """Alerting-class conditions as ``event`` records on the record plane;
    repeats of one (class, path) within ``collapse_s`` are counted, not
    re-sent, and at most ``live_cap`` distinct alerts stay live."""

    def __init__(self, store=None, collapse_s: float = 60.0, live_cap: int = 64, log=print):
        self.store, self.collapse_s, self.cap, self.log = store, collapse_s, live_cap, log
        self.live: "collections.OrderedDict[Tuple[str, str], dict]" = collections.OrderedDict()

    def raise_(self, cls: str, path: str, detail: str, now: Optional[float] = None) -> Optional[dict]:
        if cls not in ALERT_CLASSES:
            raise ValueError(f"alert class {cls!r} is not one of {ALERT_CLASSES}")
        now = time.time() if now is None else now
        key = (cls, path)
        rec = self.live.get(key)
        if rec is not None and now - rec["ts"] < self.collapse_s:
            rec["repeats"] += 1
            return None
        rec = {"kind": "event", "class": cls, "path": path, "ts": now, "sev": "critical"
               if cls == "rank_lost" else "warn", "message": detail, "repeats": 0}
        self.live[key] = rec
        self.live.move_to_end(key)
        while len(self.live) > self.cap:
            self.live.popitem(last=False)
        self.log(f"[alert] {cls} at {path}: {detail}")
        if self.store is not None:
            self.store.publish(dict(rec))
        return rec


# ----------------------------------------------------------------- failure threshold
@dataclass
class MaxFailureThreshold:
    """When ``dead >= limit_for(world)`` the run is unrecoverable: survivors
    save (``SaveReason.MaxFailureExceeded``) and stop instead of waiting for a
    re-formation that cannot complete. ``absolute`` counts ranks; ``percent``
    is a fraction of the world, clamped to [0, 1] and rounded up."""

    absolute: Optional[int] = None
    percent: Optional[float] = None

    def limit_for(self, world: int) -> int:
        if self.absolute is not None:
            return self.absolute
        p = min(max(self.percent or 0.0, 0.0), 1.0)
        return int(-(-p * world // 1))  # ceil

    def breached(self, dead: int, world: int) -> bool:
        return dead >= self.limit_for(world)
