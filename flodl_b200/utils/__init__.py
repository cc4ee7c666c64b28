"""Utilities: logging, hardware detection, flat parameter arenas, RNG."""
from . import hw, log  # noqa: F401
from .arena import ParamArena, arena_of  # noqa: F401
from .worker import CpuWorker, Rng  # noqa: F401
