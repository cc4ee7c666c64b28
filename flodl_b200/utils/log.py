"""Verbosity-gated logging (flodl/src/log.rs:39-228).

Levels: Quiet < Normal < Verbose < Debug < Trace. The level comes from
``set_verbosity`` or the ``FLODL_VERBOSITY`` environment variable (0-4 or a
name). ``msg`` prints at Normal, ``verbose``/``debug``/``trace`` at their
levels; lines carry an optional node/thread label.
"""
from __future__ import annotations

import enum
import os
import sys
import threading
import time


class Verbosity(enum.IntEnum):
    QUIET = 0
    NORMAL = 1
    VERBOSE = 2
    DEBUG = 3
    TRACE = 4


def _from_env() -> Verbosity:
    v = os.environ.get("FLODL_VERBOSITY", "1").strip().upper()
    if v.isdigit():
        return Verbosity(min(int(v), 4))
    return Verbosity[v] if v in Verbosity.__members__ else Verbosity.NORMAL


_level = _from_env()
_label = threading.local()


def set_verbosity(v) -> None:
    global _level
    _level = Verbosity(v)


def verbosity() -> Verbosity:
    return _level


def set_label(label: str) -> None:
    _label.value = label


def _emit(level: Verbosity, text: str) -> None:
    if _level < level:
        return
    lab = getattr(_label, "value", None)
    prefix = f"[{lab}] " if lab else ""
    ts = time.strftime("%H:%M:%S") if level >= Verbosity.DEBUG else ""
    sys.stderr.write(f"{ts + ' ' if ts else ''}{prefix}{text}\n")


def msg(text: str) -> None:
    _emit(Verbosity.NORMAL, text)


def verbose(text: str) -> None:
    _emit(Verbosity.VERBOSE, text)


def debug(text: str) -> None:
    _emit(Verbosity.DEBUG, text)


def trace(text: str) -> None:
    _emit(Verbosity.TRACE, text)


_seq = {"n": 0}
_seq_lock = threading.Lock()


class collective:
    """``with log.collective("all_reduce", bytes=n):`` - at Trace level,
    ENTER/EXIT lines with a per-process sequence number around a collective,
    so the first rank whose sequence diverges pins a desynchronised rank
    (reference role: the ENTER/EXIT trace around every collective,
    distributed/ddp_run/worker/sync.rs:141-227). Costs one comparison when
    Trace is off."""

    def __init__(self, name: str, **meta):
        self.name, self.meta = name, meta
        self.on = _level >= Verbosity.TRACE

    def __enter__(self):
        if self.on:
            with _seq_lock:
                _seq["n"] += 1
                self.k = _seq["n"]
            extra = " ".join(f"{k}={v}" for k, v in self.meta.items())
            _emit(Verbosity.TRACE, f"ENTER {self.name} #{self.k} {extra}".rstrip())
            self.t0 = time.perf_counter()
        return self

    def __exit__(self, et, ev, tb):
        if self.on:
            ms = (time.perf_counter() - self.t0) * 1e3
            state = "EXIT" if et is None else f"FAIL({et.__name__})"
            _emit(Verbosity.TRACE, f"{state} {self.name} #{self.k} {ms:.2f} ms")
        return False
