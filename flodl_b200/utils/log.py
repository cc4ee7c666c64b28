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
