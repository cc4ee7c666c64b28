"""Observability: training monitor, live SSE dashboard, resource timeline,
the path-keyed record plane (store, JSONL log, dashboard sink, alerts) and
the telemetry spill and shipper."""
from .monitor import Monitor, Timeline  # noqa: F401
from .records import (DashboardEmitter, DashboardSink, Leaf, RecordLog,  # noqa: F401
                      RecordStore, Reduction, Severity, build_tree)
from .telemetry import (EpochMetrics, TelemetryShipper, TimelineSpill, drain_scalars,  # noqa: F401
                        record_scalar, telemetry_dir)
