"""Cluster membership: the join window and the admission ledger.

Reference: flodl/src/distributed/membership.rs (``StartMode`` :93,
``ClusterPhase`` :238). Ranks dial in during a join window; the ledger
admits them (duplicates and late joiners are refused), decides when the world
forms, and afterwards only shrinks: a rank that dies or leaves is removed and
its partition is absorbed by the survivors.

* ``Auto``   the world forms as soon as ``expected`` members joined.
* ``Manual`` the world forms on :meth:`JoinWindow.start` (at least ``min_size``).
* ``Hybrid`` whichever comes first; at the window deadline the world forms
             with the members present if there are at least ``min_size``.
"""
from __future__ import annotations

import enum
import threading
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional


class StartMode(enum.Enum):
    Auto = "auto"
    Manual = "manual"
    Hybrid = "hybrid"


class ClusterPhase(enum.Enum):
    Joining = "joining"
    Running = "running"
    Shrinking = "shrinking"
    Finished = "finished"
    Failed = "failed"


@dataclass
class Member:
    name: str
    host: str = ""
    devices: int = 1
    joined_at: float = field(default_factory=time.monotonic)
    rank: int = -1
    alive: bool = True


class JoinWindow:
    def __init__(self, expected: int, mode: StartMode = StartMode.Auto, min_size: int = 1,
                 window_s: float = 120.0):
        if expected < 1 or min_size < 1 or min_size > expected:
            raise ValueError("need 1 <= min_size <= expected")
        self.expected, self.mode, self.min_size = expected, mode, min_size
        self.window_s = window_s
        self.opened = time.monotonic()
        self.phase = ClusterPhase.Joining
        self.members: Dict[str, Member] = {}
        self.refused: List[tuple] = []
        self.deaths: List[dict] = []
        self._lock = threading.Lock()
        self._formed = threading.Event()

    # -------------------------------------------------------------- admission
    def join(self, name: str, host: str = "", devices: int = 1) -> bool:
        with self._lock:
            if self.phase is not ClusterPhase.Joining:
                self.refused.append((name, "world already formed"))
                return False
            if name in self.members:
                self.refused.append((name, "duplicate member"))
                return False
            if len(self.members) >= self.expected:
                self.refused.append((name, "window full"))
                return False
            self.members[name] = Member(name, host, devices)
            if self.mode is not StartMode.Manual and len(self.members) == self.expected:
                self._form()
            return True

    def start(self) -> bool:
        """Manual / Hybrid start with the members present."""
        with self._lock:
            if self.phase is not ClusterPhase.Joining:
                return self.phase is ClusterPhase.Running
            if self.mode is StartMode.Auto:
                return False
            if len(self.members) < self.min_size:
                return False
            self._form()
            return True

    def poll(self) -> ClusterPhase:
        """Apply the window deadline (Hybrid forms, others fail)."""
        with self._lock:
            if self.phase is ClusterPhase.Joining and time.monotonic() - self.opened > self.window_s:
                if self.mode is StartMode.Hybrid and len(self.members) >= self.min_size:
                    self._form()
                else:
                    self.phase = ClusterPhase.Failed
            return self.phase

    def wait_formed(self, timeout: Optional[float] = None) -> bool:
        return self._formed.wait(timeout)

    def _form(self) -> None:
        # ranks in join order; a member's devices take consecutive ranks
        r = 0
        for m in sorted(self.members.values(), key=lambda m: m.joined_at):
            m.rank = r
            r += m.devices
        self.phase = ClusterPhase.Running
        self._formed.set()

    # -------------------------------------------------------------- shrinking
    @property
    def world(self) -> int:
        return sum(m.devices for m in self.members.values() if m.alive and m.rank >= 0)

    def alive(self) -> List[Member]:
        return [m for m in self.members.values() if m.alive]

    def remove(self, name: str, reason: str) -> None:
        """A member died or left: membership only shrinks."""
        with self._lock:
            m = self.members.get(name)
            if m is None or not m.alive:
                return
            m.alive = False
            self.deaths.append({"member": name, "rank": m.rank, "reason": reason,
                                "at": time.time()})
            self.phase = ClusterPhase.Shrinking if self.alive() else ClusterPhase.Failed

    def partition(self, n_items: int) -> Dict[str, range]:
        """Contiguous shares of ``n_items`` over the alive members, weighted by
        their device counts (survivors absorb a dead member's share)."""
        alive = sorted(self.alive(), key=lambda m: m.rank)
        total = sum(m.devices for m in alive)
        out, start = {}, 0
        for i, m in enumerate(alive):
            n = n_items - start if i == len(alive) - 1 else n_items * m.devices // total
            out[m.name] = range(start, start + n)
            start += n
        return out
