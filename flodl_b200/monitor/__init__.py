"""Observability: training monitor, live SSE dashboard, resource timeline."""
from .monitor import Monitor, Timeline  # noqa: F401
