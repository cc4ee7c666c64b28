"""Streaming-mode staging cascade: memory budgets, RAM sample cache, disk
stage, device sample pool, and the host dataset cache.

Reference roles: flodl/src/data/{budget.rs, sample_cache.rs, vram_pool.rs,
host_cache.rs} and the disk stage of loader.rs:370-420.

A streaming batch is assembled from per-sample reads that fall through tiers:

    VramPool (device rows, gathered in place)  ->  SampleCache (host RAM)
      ->  DiskStage (local pack file)  ->  the dataset's own ``get``

Every epoch touches each sample once in a fresh random order, so for a tier
holding K of N samples the expected hit rate is K/N whatever is kept: each
tier admits until its budget is full and never evicts (``evict`` exists for
re-partitioning between epochs).

Budget law (one place): a host tier may hold ``min(r, 0.9) x (available +
held)`` bytes, where ``available`` is ``MemAvailable`` and ``held`` what the
tier already retains (added back so the cap stays anchored to the memory the
run started with). On a unified-memory part the GPU's share of the same DRAM
(``gpu_ram_share x MemTotal``) is removed first. Device prefetch depth fills
``cap x total - used - reserve`` of VRAM with batches, clamped to
``[2, max_depth]``.
"""
from __future__ import annotations

import os
import tempfile
import threading
import warnings
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

HOST_CAP = 0.90


# ----------------------------------------------------------------- budgets
def meminfo() -> Dict[str, int]:
    out = {}
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                k, _, rest = line.partition(":")
                out[k] = int(rest.split()[0]) * 1024
    except (OSError, ValueError, IndexError):
        pass
    return out


def host_available_bytes(gpu_ram_share: Optional[float] = None, info: Optional[dict] = None) -> int:
    info = info if info is not None else meminfo()
    avail = info.get("MemAvailable", info.get("MemFree", 0))
    if gpu_ram_share:
        avail = max(0, avail - int(gpu_ram_share * info.get("MemTotal", 0)))
    return avail


def host_budget(frac: float, available: int, held: int = 0) -> int:
    """The host-RAM budget law: ``min(frac, 0.9) x (available + held)``."""
    return int(max(0.0, min(frac, HOST_CAP)) * (available + held))


def prefetch_depth(cap_frac: float, total: int, used: int, batch_bytes: int,
                   reserve: int = 0, max_depth: int = 64) -> int:
    cap = min(max(cap_frac, 0.50), 0.99)
    room = cap * total - used - reserve
    if batch_bytes <= 0:
        return 2
    return int(min(max(room // batch_bytes, 2), max_depth))


def _nbytes(rows: Sequence[torch.Tensor]) -> int:
    return sum(t.numel() * t.element_size() for t in rows)


# ----------------------------------------------------------------- RAM tier
class SampleCache:
    """Sample-keyed host cache: admit until ``budget`` bytes, no eviction."""

    def __init__(self, budget_bytes: int):
        self.budget = int(budget_bytes)
        self.held = 0
        self.slots: Dict[int, List[torch.Tensor]] = {}
        self.hits = self.misses = 0
        self._lock = threading.Lock()

    def get(self, idx: int) -> Optional[List[torch.Tensor]]:
        with self._lock:
            v = self.slots.get(idx)
            if v is None:
                self.misses += 1
            else:
                self.hits += 1
            return v

    def admit(self, idx: int, rows: List[torch.Tensor]) -> bool:
        b = _nbytes(rows)
        with self._lock:
            if idx in self.slots or self.held + b > self.budget:
                return False
            self.slots[idx] = [r.clone() for r in rows]
            self.held += b
            return True

    def evict(self, idx: int) -> None:
        with self._lock:
            v = self.slots.pop(idx, None)
            if v is not None:
                self.held -= _nbytes(v)

    def __len__(self):
        return len(self.slots)


# ----------------------------------------------------------------- disk tier
def _fs_type(path: str) -> str:
    best, fs = "", ""
    try:
        with open("/proc/mounts") as f:
            for line in f:
                parts = line.split()
                mnt = parts[1]
                if path.startswith(mnt) and len(mnt) > len(best):
                    best, fs = mnt, parts[2]
    except OSError:
        pass
    return fs


class DiskStage:
    """Append-only pack file of samples the RAM tier declined; removed on close."""

    def __init__(self, budget_bytes: int, directory: Optional[str] = None):
        d = directory or tempfile.gettempdir()
        if _fs_type(os.path.abspath(d)) in ("tmpfs", "ramfs"):
            warnings.warn(f"disk stage directory {d} is RAM-backed: staging there spends RAM")
        fd, self.path = tempfile.mkstemp(prefix="flodl_stage_", suffix=".pack", dir=d)
        self.f = os.fdopen(fd, "r+b")
        self.budget = int(budget_bytes)
        self.size = 0
        self.index: Dict[int, List[Tuple[int, tuple, str, int]]] = {}
        self.hits = 0
        self._lock = threading.Lock()

    def admit(self, idx: int, rows: List[torch.Tensor]) -> bool:
        b = _nbytes(rows)
        with self._lock:
            if idx in self.index or self.size + b > self.budget:
                return False
            entries = []
            self.f.seek(self.size)
            for r in rows:
                a = r.detach().cpu().contiguous()
                raw = a.reshape(-1).view(torch.uint8).numpy().tobytes() if a.numel() else b""
                entries.append((self.f.tell(), tuple(a.shape), str(a.dtype).replace("torch.", ""),
                                len(raw)))
                self.f.write(raw)
            self.size = self.f.tell()
            self.index[idx] = entries
            return True

    def get(self, idx: int) -> Optional[List[torch.Tensor]]:
        with self._lock:
            ent = self.index.get(idx)
            if ent is None:
                return None
            out = []
            self.f.flush()
            for off, shape, dt, n in ent:
                self.f.seek(off)
                buf = bytearray(self.f.read(n))
                t = torch.frombuffer(buf, dtype=torch.uint8) if n else torch.empty(0, dtype=torch.uint8)
                out.append(t.view(getattr(torch, dt)).reshape(shape))
            self.hits += 1
            return out

    def close(self) -> None:
        try:
            self.f.close()
            os.unlink(self.path)
        except OSError:
            pass

    def __del__(self):
        self.close()


# ----------------------------------------------------------------- device tier
class VramPool:
    """Device-resident sample rows; a batch gathers its hits in place and
    uploads only the misses. Rows enter from batches uploaded anyway."""

    def __init__(self, capacity: int, row_shapes: List[tuple], dtypes: List[torch.dtype], device):
        self.capacity = int(capacity)
        self.device = torch.device(device)
        self.bufs = [torch.empty((self.capacity, *s), dtype=d, device=self.device)
                     for s, d in zip(row_shapes, dtypes)]
        self.slot_of = torch.full((0,), -1, dtype=torch.long)
        self.used = 0
        self.hits = self.misses = 0

    def _ensure(self, n: int) -> None:
        if self.slot_of.numel() < n:
            grow = torch.full((n - self.slot_of.numel(),), -1, dtype=torch.long)
            self.slot_of = torch.cat([self.slot_of, grow])

    def lookup(self, idx: torch.Tensor) -> torch.Tensor:
        """Pool slot of each sample (-1 = miss)."""
        self._ensure(int(idx.max()) + 1 if idx.numel() else 0)
        s = self.slot_of[idx]
        h = int((s >= 0).sum())
        self.hits += h
        self.misses += idx.numel() - h
        return s

    def gather(self, slots: torch.Tensor) -> List[torch.Tensor]:
        sd = slots.to(self.device, non_blocking=True)
        return [b.index_select(0, sd) for b in self.bufs]

    def admit(self, idx: torch.Tensor, rows: List[torch.Tensor]) -> int:
        free = self.capacity - self.used
        if free <= 0 or idx.numel() == 0:
            return 0
        k = min(free, idx.numel())
        take = torch.arange(self.used, self.used + k)
        td = take.to(self.device, non_blocking=True)
        for b, r in zip(self.bufs, rows):
            b.index_copy_(0, td, r[:k])
        self._ensure(int(idx[:k].max()) + 1)
        self.slot_of[idx[:k]] = take
        self.used += k
        return k


# ----------------------------------------------------------------- host dataset cache
def publish_atomically(tmp: str, dst: str) -> None:
    os.replace(tmp, dst)


def resolve_cached(root: str, dataset: str, name: str, is_valid: Callable[[str], bool],
                   fetch: Callable[[str], None], cache_root: Optional[str] = None) -> str:
    """Path of a dataset file: the read-only source root when it has a valid
    copy, else the writable host cache, acquiring it there once through
    ``fetch(destination)`` (written to a temporary name, then renamed)."""
    src = os.path.join(root, dataset, name)
    if os.path.exists(src) and is_valid(src):
        return src
    base = cache_root or os.environ.get("FLODL_HOST_CACHE",
                                        os.path.join(os.path.expanduser("~"), ".cache", "flodl"))
    dst = os.path.join(base, dataset, name)
    if os.path.exists(dst) and is_valid(dst):
        return dst
    os.makedirs(os.path.dirname(dst), exist_ok=True)
    tmp = dst + f".part{os.getpid()}"
    fetch(tmp)
    if not is_valid(tmp):
        os.unlink(tmp)
        raise RuntimeError(f"fetched {name} for {dataset} failed validation")
    publish_atomically(tmp, dst)
    return dst
