"""Telemetry plane: node-local timeline spill and the shipper that mirrors it
to shared storage; epoch metrics and the scalar drain.

Reference roles: flodl/src/monitor/spill.rs, shipper.rs and metrics.rs.

* :class:`TimelineSpill` appends every timeline sample and event to a bounded
  JSONL ring (``timeline.log`` + ``timeline.log.1``) in
  ``~/.flodl/telemetry/<label>-<UTC stamp>-<pid>/`` with a ``meta.json``
  (host, pid, start) beside it. It runs on its own thread; I/O errors are
  warned once and never reach training.
* :class:`TelemetryShipper` tail-follows that directory: ``*.log`` files are
  streams (a byte offset and inode per file; new bytes are appended to
  ``<name>.partial`` at the destination; when the active segment's inode
  changed, the unshipped tail is recovered from ``.log.1`` first), other files are copied
  whole through a temporary name. ``finish`` ships the residue and renames
  every ``.partial`` to its final name, waiting a bounded time.
* :class:`EpochMetrics`, :func:`record_scalar` / :func:`drain_scalars` - the
  per-epoch aggregation vocabulary the monitor renders.
"""
from __future__ import annotations

import json
import os
import shutil
import socket
import threading
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional


def telemetry_dir(label: str, root: Optional[str] = None) -> str:
    base = root or os.path.join(os.path.expanduser("~"), ".flodl", "telemetry")
    stamp = time.strftime("%Y%m%dT%H%M%SZ", time.gmtime())
    return os.path.join(base, f"{label}-{stamp}-{os.getpid()}")


class TimelineSpill:
    def __init__(self, directory: str, segment_bytes: int = 8 << 20, flush_s: float = 1.0):
        self.dir = directory
        self.seg = segment_bytes
        self.flush_s = flush_s
        self._buf: List[dict] = []
        self._lock = threading.Lock()
        self._warned = False
        self._stop = threading.Event()
        try:
            os.makedirs(directory, exist_ok=True)
            with open(os.path.join(directory, "meta.json"), "w") as f:
                json.dump({"host": socket.gethostname(), "pid": os.getpid(), "start": time.time()}, f)
        except OSError as e:
            self._warn(e)
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    @property
    def path(self) -> str:
        return os.path.join(self.dir, "timeline.log")

    def _warn(self, e):
        if not self._warned:
            self._warned = True
            print(f"telemetry spill: {e} (further errors are silent)")

    def sample(self, rec: dict) -> None:
        with self._lock:
            self._buf.append(rec)

    def event(self, kind: str, **fields) -> None:
        self.sample({"t": time.time(), "k": kind, **fields})

    def _flush(self) -> None:
        with self._lock:
            buf, self._buf = self._buf, []
        if not buf:
            return
        try:
            if os.path.exists(self.path) and os.path.getsize(self.path) > self.seg:
                os.replace(self.path, self.path + ".1")
            with open(self.path, "a") as f:
                for r in buf:
                    f.write(json.dumps(r) + "\n")
        except OSError as e:
            self._warn(e)

    def _run(self):
        while not self._stop.wait(self.flush_s):
            self._flush()

    def close(self) -> None:
        self._stop.set()
        self._t.join(timeout=5)
        self._flush()


class TelemetryShipper:
    def __init__(self, src: str, dst: str, interval_s: float = 2.0):
        self.src, self.dst, self.interval = src, dst, interval_s
        self.offsets: Dict[str, int] = {}
        self.inodes: Dict[str, int] = {}
        self.copied: Dict[str, float] = {}
        self.warned = set()
        self._ship_lock = threading.Lock()  # the tick thread and finish() never ship at once
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def _warn(self, name, e):
        if name not in self.warned:
            self.warned.add(name)
            print(f"telemetry shipper: {name}: {e} (retrying)")

    def _append(self, name: str, data: bytes) -> None:
        with open(os.path.join(self.dst, name + ".partial"), "ab") as f:
            f.write(data)

    def ship_once(self) -> None:
        with self._ship_lock:
            self._ship_once()

    def _ship_once(self) -> None:
        try:
            os.makedirs(self.dst, exist_ok=True)
            names = sorted(os.listdir(self.src))
        except OSError as e:
            self._warn("dir", e)
            return
        for n in names:
            p = os.path.join(self.src, n)
            try:
                if n.endswith(".log"):
                    off = self.offsets.get(n, 0)
                    st = os.stat(p)
                    ino = self.inodes.get(n)
                    if ino is not None and st.st_ino != ino:
                        # rotated since the last tick: finish the old segment
                        # (now the .log.1 sibling) before following the new one
                        rot = p + ".1"
                        if os.path.exists(rot) and os.stat(rot).st_ino == ino:
                            with open(rot, "rb") as f:
                                f.seek(off)
                                self._append(n, f.read())
                        off = 0
                    self.inodes[n] = st.st_ino
                    if st.st_size > off:
                        with open(p, "rb") as f:
                            f.seek(off)
                            data = f.read(st.st_size - off)
                        self._append(n, data)
                        off += len(data)
                    self.offsets[n] = off
                elif n.endswith(".log.1"):
                    continue
                else:
                    m = os.path.getmtime(p)
                    if self.copied.get(n) != m:
                        tmp = os.path.join(self.dst, n + ".tmp")
                        shutil.copyfile(p, tmp)
                        os.replace(tmp, os.path.join(self.dst, n))
                        self.copied[n] = m
            except OSError as e:
                self._warn(n, e)

    def _run(self):
        while not self._stop.wait(self.interval):
            self.ship_once()

    def finish(self, timeout_s: float = 30.0) -> bool:
        """Final ship and publish (.partial -> final name). False if the
        destination stalled past ``timeout_s`` (the thread is left detached)."""
        self._stop.set()
        done = threading.Event()

        def final():
            self._t.join()
            self.ship_once()
            for n in list(self.offsets):
                part = os.path.join(self.dst, n + ".partial")
                if os.path.exists(part):
                    os.replace(part, os.path.join(self.dst, n))
            done.set()

        threading.Thread(target=final, daemon=True).start()
        return done.wait(timeout_s)


# ----------------------------------------------------------------- epoch metrics
@dataclass
class EpochMetrics:
    epoch: int
    loss: Optional[float] = None
    throughput: Optional[float] = None          # samples / s
    batch_share: List[float] = field(default_factory=list)
    scalars: Dict[str, float] = field(default_factory=dict)


_SCALARS: Dict[str, List[float]] = {}
_SCALAR_LOCK = threading.Lock()


def record_scalar(name: str, value: float) -> None:
    with _SCALAR_LOCK:
        _SCALARS.setdefault(name, []).append(float(value))


def drain_scalars() -> Dict[str, float]:
    """Means of everything recorded since the last drain (then cleared)."""
    with _SCALAR_LOCK:
        out = {k: sum(v) / len(v) for k, v in _SCALARS.items() if v}
        _SCALARS.clear()
    return out
