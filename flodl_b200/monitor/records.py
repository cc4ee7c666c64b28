"""Path-keyed record plane: tree builder, JSONL log, live store, dashboard sink.

Reference roles: flodl/src/monitor/record.rs (record tree and reductions),
record_log.rs (bounded per-node JSONL), record_store.rs (latest state and
history per path, one delivery predicate for stream and history),
event_lane.rs (alerts) and distributed/dashboard_sink.rs (controller-side
endpoint for rank frames).

Every monitored node is one record addressed by a ``/``-separated path:
``root``, ``root/rank3`` or ``root/<host>/rank3``. A leaf (a rank) carries raw
values; an interior node carries the same fields aggregated over its DIRECT
children. ``Mean`` is weighted by realized work (samples), so a hierarchical
mean equals the flat one; a key no child reported is absent, never zero; a
zero-work child is excluded from means. Core keys have fixed reductions
(``throughput`` and ``batch_share`` sum, ``loss`` mean, ``data_starve`` and
``compute_only_ms`` max); other keys use the declared reduction (default mean).
"""
from __future__ import annotations

import collections
import enum
import json
import os
import queue
import socket
import struct
import threading
import time
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Sequence, Tuple


class Severity(enum.Enum):
    Info = "info"
    Warn = "warn"
    Critical = "critical"


class Reduction(enum.Enum):
    Mean = "mean"
    Sum = "sum"
    Max = "max"
    Min = "min"
    Last = "last"

    def reduce(self, contribs: Sequence[Tuple[float, float]]) -> Optional[float]:
        """Roll (value, work) pairs of the direct children into one value."""
        if not contribs:
            return None
        vals = [v for v, _ in contribs]
        if self is Reduction.Sum:
            return sum(vals)
        if self is Reduction.Max:
            return max(vals)
        if self is Reduction.Min:
            return min(vals)
        if self is Reduction.Last:  # the child with the most work
            return max(contribs, key=lambda c: c[1])[0]
        w = sum(wt for _, wt in contribs if wt > 0)
        if w <= 0:
            return None
        return sum(v * wt for v, wt in contribs if wt > 0) / w


_CORE = {"throughput": Reduction.Sum, "batch_share": Reduction.Sum, "loss": Reduction.Mean,
         "data_starve": Reduction.Max, "compute_only_ms": Reduction.Max}
# resource fields: utilisation means, memory sums, peaks max
_RES = {"gpu_util": Reduction.Mean, "vram_used_mb": Reduction.Sum, "vram_total_mb": Reduction.Sum,
        "gpu_util_max": Reduction.Max, "vram_used_max_mb": Reduction.Max,
        "ram_used_mb": Reduction.Sum, "power_w": Reduction.Sum, "temp_c": Reduction.Max}


def core_reduction(key: str) -> Optional[Reduction]:
    return _CORE.get(key)


def reduction_for(key: str, user: Dict[str, Reduction]) -> Reduction:
    return _CORE.get(key) or _RES.get(key) or user.get(key, Reduction.Mean)


@dataclass
class Leaf:
    path: List[str]                      # segments below root, leaf id last
    work: float = 0.0
    metrics: Dict[str, float] = field(default_factory=dict)
    res: Dict[str, float] = field(default_factory=dict)
    device: Optional[int] = None
    alive: bool = True
    label: Optional[str] = None


@dataclass
class NodeRecord:
    path: List[str]
    work: float
    metrics: Dict[str, float]
    res: Dict[str, float]
    children: List["NodeRecord"] = field(default_factory=list)
    device: Optional[int] = None
    alive: bool = True
    label: Optional[str] = None
    epoch_complete: bool = False

    def is_leaf(self) -> bool:
        return not self.children

    @property
    def path_str(self) -> str:
        return "/".join(self.path)

    def to_record_json(self, ts: float, tick: Optional[int] = None, epoch: Optional[int] = None,
                       sev: Severity = Severity.Info) -> dict:
        r = {"kind": "node", "path": self.path_str, "ts": ts, "sev": sev.value, "work": self.work,
             "metrics": dict(self.metrics), "res": dict(self.res),
             "epoch_complete": self.epoch_complete}
        if tick is not None:
            r["tick"] = tick
        if epoch is not None:
            r["epoch"] = epoch
        if self.is_leaf():
            r["alive"] = self.alive
            if self.device is not None:
                r["device"] = self.device
        else:
            r["children"] = len(self.children)
            r["alive"] = sum(c.alive for c in self.children)
        if self.label:
            r["label"] = self.label
        return r

    def flat_records(self, ts: float, tick=None, epoch=None) -> List[dict]:
        out = [self.to_record_json(ts, tick, epoch)]
        for c in self.children:
            out += c.flat_records(ts, tick, epoch)
        return out


def cohort_tiering(hosts: Sequence[str]) -> Tuple[bool, bool]:
    """(multi_host, root_only) for one rank per entry of ``hosts``."""
    named = {h for h in hosts if h}
    multi = len(named) > 1
    return multi, len(hosts) == 1 and not multi


def leaf_path_segments(rank: int, hosts: Sequence[str]) -> List[str]:
    multi, root_only = cohort_tiering(hosts)
    if root_only:
        return []
    host = hosts[rank] if rank < len(hosts) else ""
    return ([host] if multi and host else []) + [f"rank{rank}"]


def rank_record_path(rank: int, hosts: Sequence[str]) -> str:
    return "/".join(["root"] + leaf_path_segments(rank, hosts))


def build_tree(leaves: Sequence[Leaf], user: Optional[Dict[str, Reduction]] = None,
               epoch_complete: bool = False) -> NodeRecord:
    user = user or {}

    def build(prefix: List[str], entries: List[Tuple[List[str], Leaf]]) -> NodeRecord:
        here = [l for rest, l in entries if not rest]
        if here and len(entries) == 1:
            l = here[0]
            return NodeRecord(prefix, l.work, dict(l.metrics), dict(l.res), [], l.device, l.alive,
                              l.label, epoch_complete)
        groups: Dict[str, List[Tuple[List[str], Leaf]]] = collections.OrderedDict()
        for rest, l in entries:
            if rest:
                groups.setdefault(rest[0], []).append((rest[1:], l))
        kids = [build(prefix + [k], g) for k, g in groups.items()]
        work = sum(c.work for c in kids)
        metrics, res = {}, {}
        for attr, out in (("metrics", metrics), ("res", res)):
            keys = sorted({k for c in kids for k in getattr(c, attr)})
            for k in keys:
                contribs = [(getattr(c, attr)[k], c.work) for c in kids if k in getattr(c, attr)]
                v = reduction_for(k, user).reduce(contribs)
                if v is not None:
                    out[k] = v
        return NodeRecord(prefix, work, metrics, res, kids, None, any(c.alive for c in kids),
                          None, epoch_complete)

    return build(["root"], [(list(l.path), l) for l in leaves])


def event_record(path: str, kind: str, message: str, sev: Severity = Severity.Info,
                 **fields) -> dict:
    """A ``log``/``event`` record: alerts and discrete events (the alert lane)."""
    return {"kind": kind, "path": path, "ts": time.time(), "sev": sev.value, "message": message,
            **fields}


# ----------------------------------------------------------------- delivery predicate
def _under(path: str, p: str) -> bool:
    return path == p or path.startswith(p + "/")


def delivers(record: dict, p: str) -> bool:
    """What a subscriber at ``p`` receives (and ``history(p)`` returns): node
    records of ``p`` and its direct children; log/event records from anywhere
    under ``p`` (an alert must reach a root viewer)."""
    path = record.get("path", "")
    if record.get("kind") == "node":
        if path == p:
            return True
        return path.startswith(p + "/") and "/" not in path[len(p) + 1:]
    return _under(path, p)


# ----------------------------------------------------------------- JSONL log
class RecordLog:
    """Append-only JSONL per node: ``root/host/rank0`` -> ``<dir>/root/host/rank0.log``.
    Bounded: each node keeps at most ``segments`` files of ``segment_bytes``;
    the oldest is dropped on rotation. I/O errors are swallowed (warned once
    per node): observability must never fail a training run."""

    def __init__(self, directory: str, segment_bytes: int = 4 << 20, segments: int = 4):
        self.dir, self.seg_bytes, self.segments = directory, segment_bytes, segments
        self._warned = set()
        self._lock = threading.Lock()

    def _file(self, path: str, i: int = 0) -> str:
        base = os.path.join(self.dir, *path.split("/")) + ".log"
        return base if i == 0 else f"{base}.{i}"

    def append(self, record: dict) -> None:
        path = record.get("path", "root")
        line = json.dumps(record) + "\n"
        with self._lock:
            try:
                f0 = self._file(path)
                os.makedirs(os.path.dirname(f0), exist_ok=True)
                if os.path.exists(f0) and os.path.getsize(f0) + len(line) > self.seg_bytes:
                    for i in range(self.segments - 1, 0, -1):
                        src = self._file(path, i - 1)
                        if os.path.exists(src):
                            os.replace(src, self._file(path, i))
                with open(f0, "a") as f:
                    f.write(line)
            except OSError as e:
                if path not in self._warned:
                    self._warned.add(path)
                    print(f"record log: {path}: {e} (further errors for this node are silent)")

    def tail(self, path: str, n: int) -> List[dict]:
        """The last ``n`` records of a node (newest last), across segments."""
        out: List[dict] = []
        for i in range(self.segments):
            fn = self._file(path, i)
            if not os.path.exists(fn):
                continue
            try:
                with open(fn) as f:
                    lines = f.readlines()
            except OSError:
                continue
            out = [json.loads(x) for x in lines if x.strip()] + out
            if len(out) >= n:
                break
        return out[-n:] if n > 0 else []


# ----------------------------------------------------------------- live store
class RecordStore:
    """Latest node record per path, a bounded history, and SSE subscribers."""

    def __init__(self, history: int = 4096, log: Optional[RecordLog] = None):
        self.latest: Dict[str, dict] = {}
        self.hist: Deque[dict] = collections.deque(maxlen=history)
        self.log = log
        self._subs: List[Tuple[str, "queue.Queue[dict]"]] = []
        self._lock = threading.Lock()

    def publish(self, record: dict) -> None:
        with self._lock:
            if record.get("kind") == "node":
                self.latest[record["path"]] = record
            self.hist.append(record)
            subs = list(self._subs)
        if self.log is not None:
            self.log.append(record)
        for p, q in subs:
            if delivers(record, p):
                try:
                    q.put_nowait(record)
                except queue.Full:
                    pass

    def publish_tree(self, tree: NodeRecord, tick=None, epoch=None) -> None:
        for r in tree.flat_records(time.time(), tick, epoch):
            self.publish(r)

    def paths(self) -> List[str]:
        with self._lock:
            return sorted(self.latest)

    def node(self, p: str) -> dict:
        """Latest record at ``p`` plus one per direct child."""
        with self._lock:
            kids = [r for q, r in self.latest.items()
                    if q.startswith(p + "/") and "/" not in q[len(p) + 1:]]
            return {"node": self.latest.get(p), "children": sorted(kids, key=lambda r: r["path"])}

    def history(self, p: str, n: int = 256) -> List[dict]:
        if n <= 0:
            return []
        with self._lock:
            return [r for r in self.hist if delivers(r, p)][-n:]

    def subscribe(self, p: str) -> "queue.Queue[dict]":
        q: "queue.Queue[dict]" = queue.Queue(maxsize=4096)
        with self._lock:
            self._subs.append((p, q))
        return q

    def unsubscribe(self, q) -> None:
        with self._lock:
            self._subs = [(p, x) for p, x in self._subs if x is not q]


# ----------------------------------------------------------------- dashboard sink
MAGIC_DASH = 0x464C4442  # "FLDB": rank -> controller record frames
K_RECORD = 1


class DashboardSink:
    """Controller-side endpoint: ranks send signed frames whose payload is one
    JSON record (or a list); each is published into a :class:`RecordStore`.
    ``port=None`` serves connections handed over by the port mux (``adopt``)."""

    def __init__(self, store: RecordStore, key: bytes, host: str = "127.0.0.1",
                 port: Optional[int] = 0):
        self.store, self.key = store, key
        self.rejected = 0
        self.srv = None
        self.port = None
        if port is not None:
            self.srv = socket.socket()
            self.srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            self.srv.bind((host, port))
            self.srv.listen(64)
            self.port = self.srv.getsockname()[1]
            threading.Thread(target=self._accept, daemon=True).start()

    def _accept(self):
        while True:
            try:
                c, _ = self.srv.accept()
            except OSError:
                return
            self.adopt(c)

    def adopt(self, c: socket.socket) -> None:
        threading.Thread(target=self._serve, args=(c,), daemon=True).start()

    def _serve(self, c: socket.socket) -> None:
        from ..parallel.cpu_reduce import recv_frame
        try:
            while True:
                kind, _, payload = recv_frame(c, self.key, magic=MAGIC_DASH, max_frame=16 << 20)
                if kind != K_RECORD:
                    raise ConnectionError("unexpected frame kind")
                recs = json.loads(payload.decode())
                for r in recs if isinstance(recs, list) else [recs]:
                    if isinstance(r, dict) and isinstance(r.get("path"), str):
                        self.store.publish(r)
        except (ConnectionError, OSError, ValueError):
            self.rejected += 1
        finally:
            c.close()

    def close(self) -> None:
        if self.srv is not None:
            self.srv.close()


class DashboardEmitter:
    """Rank side: ship records to the controller's :class:`DashboardSink`."""

    def __init__(self, host: str, port: int, key: bytes):
        self.key = key
        self.sock = socket.create_connection((host, port), timeout=30)
        self.lock = threading.Lock()

    def emit(self, records) -> None:
        from ..parallel.cpu_reduce import send_frame
        send_frame(self.sock, self.key, K_RECORD, 0, json.dumps(records).encode(), self.lock,
                   magic=MAGIC_DASH)

    def close(self) -> None:
        self.sock.close()
