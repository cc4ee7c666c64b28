"""GPU runtime wrappers: device queries, memory statistics, events, streams.

Reference roles: flodl/src/tensor/{cuda.rs, cuda_event.rs, cuda_stream.rs}
and the shim's device/memory queries (flodl-sys/ops_nn.cpp:603-1060).
``StreamGuard`` makes a stream current for a scope and restores the previous
one (also on exceptions); streams come from a per-device round-robin pool so
repeated side streams do not multiply.
"""
from __future__ import annotations

import threading
from typing import Dict, List, Optional

import torch


def gpu_available() -> bool:
    return torch.cuda.is_available()


def device_count() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def device_name(i: int = 0) -> str:
    return torch.cuda.get_device_name(i)


def compute_capability(i: int = 0) -> tuple:
    return torch.cuda.get_device_capability(i)


def arch(i: int = 0) -> str:
    major, minor = compute_capability(i)
    return f"sm_{major}{minor}"


def memory_stats(i: int = 0) -> Dict[str, int]:
    """Active / reserved bytes now and at peak, plus the device's free/total."""
    free, total = torch.cuda.mem_get_info(i)
    return {"allocated": torch.cuda.memory_allocated(i), "reserved": torch.cuda.memory_reserved(i),
            "peak_allocated": torch.cuda.max_memory_allocated(i),
            "peak_reserved": torch.cuda.max_memory_reserved(i), "free": free, "total": total}


def reset_peak_stats(i: int = 0) -> None:
    torch.cuda.reset_peak_memory_stats(i)


def empty_cache() -> None:
    torch.cuda.empty_cache()


def synchronize(i: Optional[int] = None) -> None:
    torch.cuda.synchronize(i)


class CudaEvent:
    """Timing event: ``record()`` on a stream, ``elapsed_ms(other)``."""

    def __init__(self, timing: bool = True):
        self.e = torch.cuda.Event(enable_timing=timing)

    def record(self, stream: Optional[torch.cuda.Stream] = None) -> "CudaEvent":
        self.e.record(stream)
        return self

    def synchronize(self) -> None:
        self.e.synchronize()

    def query(self) -> bool:
        return self.e.query()

    def elapsed_ms(self, end: "CudaEvent") -> float:
        return self.e.elapsed_time(end.e)


class _StreamPool:
    def __init__(self, size: int = 4):
        self.size = size
        self.pools: Dict[int, List[torch.cuda.Stream]] = {}
        self.next: Dict[int, int] = {}
        self.lock = threading.Lock()

    def get(self, device: int) -> torch.cuda.Stream:
        with self.lock:
            pool = self.pools.setdefault(device, [])
            if len(pool) < self.size:
                pool.append(torch.cuda.Stream(device))
                return pool[-1]
            i = self.next.get(device, 0)
            self.next[device] = (i + 1) % self.size
            return pool[i]


_POOL = _StreamPool()


def stream_from_pool(device: int = 0) -> torch.cuda.Stream:
    return _POOL.get(device)


class StreamGuard:
    """``with StreamGuard(s):`` runs the scope on ``s`` and restores the
    previous current stream afterwards."""

    def __init__(self, stream: torch.cuda.Stream):
        self.stream = stream
        self.prev = None

    def __enter__(self):
        self.prev = torch.cuda.current_stream(self.stream.device)
        torch.cuda.set_stream(self.stream)
        return self.stream

    def __exit__(self, *exc):
        torch.cuda.set_stream(self.prev)
        return False
