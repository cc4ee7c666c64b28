"""Cluster coordinator pieces: progressive epoch dispatch, window ledger,
callback-role election and the alert lane.

Reference roles: flodl/src/distributed/chunk_pool.rs (spans, cursors,
stealing, forfeit, coverage), cluster_coordinator/window_ledger.rs,
callback_roles.rs and alerts.rs.

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
    def __init__(self, epoch: int, total: int, spans: Sequence[int]):
        if sum(spans) != total:
            raise ValueError("spans must cover the epoch exactly")
        self.epoch, self.total = epoch, total
        self.start: List[int] = []
        acc = 0
        for s in spans:
            self.start.append(acc)
            acc += s
        self.cursor = list(self.start)                       # owner's front
        self.end = [a + s for a, s in zip(self.start, spans)]  # thieves move this down
        self.reclaimed: Deque[Tuple[int, int]] = collections.deque()
        self.outstanding: Dict[int, List[Tuple[int, int]]] = {r: [] for r in range(len(spans))}
        self.completed = 0
        self.done_samples: Dict[int, int] = {r: 0 for r in range(len(spans))}
        self.t0 = time.monotonic()

    @staticmethod
    def equal(epoch: int, total: int, world: int) -> "ChunkPool":
        return ChunkPool(epoch, total, spans_from_throughput(total, [1.0] * world))

    # ------------------------------------------------------------ views
    def residue(self, rank: int) -> int:
        return self.end[rank] - self.cursor[rank]

    def reservation(self, rank: int) -> Tuple[int, int]:
        return self.cursor[rank], self.residue(rank)

    def remaining(self) -> int:
        return sum(self.residue(r) for r in range(len(self.cursor))) + sum(n for _, n in self.reclaimed)

    def in_flight(self, rank: int) -> int:
        return sum(n for _, n in self.outstanding[rank])

    def is_epoch_done(self) -> bool:
        return self.remaining() == 0 and all(not v for v in self.outstanding.values())

    def epoch_elapsed_ms(self) -> float:
        return (time.monotonic() - self.t0) * 1e3

    # ------------------------------------------------------------ dispatch
    def take_chunk(self, size: int, rank: int) -> Optional[Tuple[int, int]]:
        if size <= 0:
            return None
        if self.reclaimed:                       # close coverage holes first
            off, n = self.reclaimed.popleft()
            k = min(n, size)
            if k < n:
                self.reclaimed.appendleft((off + k, n - k))
            chunk = (off, k)
        elif self.residue(rank) > 0:             # own span, front to back
            off = self.cursor[rank]
            k = min(size, self.residue(rank))
            self.cursor[rank] += k
            chunk = (off, k)
        else:                                    # steal the tail of the largest residue
            donor = max(range(len(self.cursor)), key=self.residue)
            if self.residue(donor) <= 0:
                return None
            k = min(size, self.residue(donor))
            self.end[donor] -= k
            chunk = (self.end[donor], k)
        self.outstanding[rank].append(chunk)
        return chunk

    def rollback_take(self, rank: int, offset: int, size: int) -> None:
        """Undo the rank's newest take (a dispatch whose send failed)."""
        out = self.outstanding[rank]
        if not out or out[-1] != (offset, size):
            raise ValueError("rollback must name the rank's newest outstanding chunk")
        out.pop()
        if self.cursor[rank] == offset + size and self.start[rank] <= offset:
            self.cursor[rank] = offset
        else:
            self.reclaimed.appendleft((offset, size))

    def mark_completed(self, rank: int, samples: int) -> None:
        out = self.outstanding[rank]
        left = samples
        while left > 0 and out:
            off, n = out[0]
            if n <= left:
                out.pop(0)
                left -= n
            else:
                out[0] = (off + left, n - left)
                left = 0
        done = samples - left  # a falsely-dead rank reporting late is clamped
        self.completed += done
        self.done_samples[rank] += done

    def forfeit(self, rank: int) -> int:
        """A dead rank: its outstanding chunks and unassigned span return to
        the pool for the survivors. Returns the reclaimed sample count."""
        n = 0
        for off, k in self.outstanding[rank]:
            self.reclaimed.append((off, k))
            n += k
        self.outstanding[rank] = []
        if self.residue(rank) > 0:
            self.reclaimed.append((self.cursor[rank], self.residue(rank)))
            n += self.residue(rank)
            self.cursor[rank] = self.end[rank]
        return n

    # ------------------------------------------------------------ coverage (resume)
    def uncovered_ranges(self) -> List[Tuple[int, int]]:
        """(offset, length) ranges not yet dispatched-and-completed."""
        rs = [(self.cursor[r], self.residue(r)) for r in range(len(self.cursor)) if self.residue(r)]
        rs += [c for v in self.outstanding.values() for c in v] + list(self.reclaimed)
        rs.sort()
        merged: List[Tuple[int, int]] = []
        for off, n in rs:
            if merged and merged[-1][0] + merged[-1][1] >= off:
                o, m = merged[-1]
                merged[-1] = (o, max(o + m, off + n) - o)
            else:
                merged.append((off, n))
        return merged

    @staticmethod
    def from_coverage(epoch: int, total: int, world: int,
                      uncovered: Sequence[Tuple[int, int]]) -> "ChunkPool":
        p = ChunkPool(epoch, total, [0] * (world - 1) + [total])
        p.cursor = list(p.end)  # every span consumed; only the holes remain
        p.reclaimed = collections.deque(sorted(uncovered))
        p.completed = total - sum(n for _, n in uncovered)
        return p


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
