"""Graph profiling and visualisation: per-node device timing, heatmap, plots,
background snapshots.

Reference roles: flodl/src/graph/profile.rs:274-530 (per-node timing through a
pool of GPU events, per-level wall clock and parallelism, statistics over
samples, timing trends), heatmap.rs (SVG heatmap of node times), plot.rs
(HTML plots, CSV trend export, training log) and snapshot.rs (CPU copy of the
model for a background save).

Timing does not synchronise per node: each node's launch is bracketed by two
CUDA events from a pool that is reused across forwards, and the durations are
resolved once, after the forward, with one synchronisation. On CPU the same
brackets use the host clock.
"""
from __future__ import annotations

import html
import json
import threading
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch


# ----------------------------------------------------------------- event pool
class EventPool:
    """Reusable timing events; ``mark()`` hands out the next one."""

    def __init__(self, cuda: bool):
        self.cuda = cuda
        self._events: List = []
        self._next = 0

    def reset(self) -> None:
        self._next = 0

    def mark(self):
        if not self.cuda:
            t = time.perf_counter()
            self._next += 1
            return t
        if self._next == len(self._events):
            self._events.append(torch.cuda.Event(enable_timing=True))
        e = self._events[self._next]
        self._next += 1
        e.record()
        return e

    def elapsed_s(self, a, b) -> float:
        return (b - a) if not self.cuda else a.elapsed_time(b) / 1e3


@dataclass
class NodeTiming:
    id: str
    tag: str
    duration: float      # seconds
    level: int


@dataclass
class LevelTiming:
    index: int
    wall_clock: float
    sum_nodes: float
    num_nodes: int

    def parallelism(self) -> float:
        return self.sum_nodes / self.wall_clock if self.wall_clock > 0 else 1.0


@dataclass
class Profile:
    total: float
    levels: List[LevelTiming]
    nodes: List[NodeTiming]
    source: str           # "cuda_events" or "host_clock"

    def timing(self, tag: str) -> float:
        return sum(n.duration for n in self.nodes if n.tag == tag or n.id == tag)

    def to_json(self) -> dict:
        return {"total_s": self.total, "source": self.source,
                "levels": [l.__dict__ for l in self.levels], "nodes": [n.__dict__ for n in self.nodes]}


@dataclass
class NodeStat:
    id: str
    tag: str
    level: int
    min: float
    mean: float
    max: float


@dataclass
class ProfileStats:
    source: str
    structural_hash: str
    samples: int
    total_min: float
    total_mean: float
    nodes: List[NodeStat] = field(default_factory=list)


class GraphProfiler:
    """Collects one :class:`Profile` per forward of a graph."""

    def __init__(self, graph, max_samples: int = 256):
        self.g = graph
        self.cuda = torch.cuda.is_available() and any(
            p.is_cuda for p in graph.parameters()) if hasattr(graph, "parameters") else False
        self.pool = EventPool(self.cuda)
        self.samples: List[Profile] = []
        self.max_samples = max_samples
        self._marks: List[Tuple[int, object, object]] = []
        self._level_marks: Dict[int, List] = {}
        self._t0 = self._t1 = None
        self._collected: Dict[str, List[float]] = {}
        self._history: Dict[str, List[float]] = {}

    # called by Graph.forward
    def begin(self) -> None:
        self.pool.reset()
        self._marks = []
        self._level_marks = {}
        self._t0 = self.pool.mark()

    def node_start(self):
        return self.pool.mark()

    def node_end(self, ni: int, start, level: int) -> None:
        end = self.pool.mark()
        self._marks.append((ni, start, end))
        lm = self._level_marks.setdefault(level, [start, end])
        lm[1] = end

    def end(self) -> Profile:
        self._t1 = self.pool.mark()
        if self.cuda:
            torch.cuda.synchronize()
        el = self.pool.elapsed_s
        tags = {}
        for t, ref in self.g.tag_names.items():
            tags.setdefault(ref.node_id, t)
        lvl_of = {ni: li for li, lvl in enumerate(self.g.levels) for ni in lvl}
        nodes = []
        for ni, a, b in self._marks:
            n = self.g._node_list[ni]
            nodes.append(NodeTiming(n.id, tags.get(n.id, n.id), el(a, b), lvl_of.get(ni, 0)))
        levels = []
        for li in sorted(self._level_marks):
            a, b = self._level_marks[li]
            ns = [x for x in nodes if x.level == li]
            levels.append(LevelTiming(li, el(a, b), sum(x.duration for x in ns), len(ns)))
        prof = Profile(el(self._t0, self._t1), levels, nodes,
                       "cuda_events" if self.cuda else "host_clock")
        self.samples.append(prof)
        if len(self.samples) > self.max_samples:
            self.samples.pop(0)
        return prof

    def stats(self) -> Optional[ProfileStats]:
        if not self.samples:
            return None
        per: Dict[str, List[NodeTiming]] = {}
        for p in self.samples:
            for n in p.nodes:
                per.setdefault(n.id, []).append(n)
        nodes = [NodeStat(k, v[0].tag, v[0].level, min(x.duration for x in v),
                          sum(x.duration for x in v) / len(v), max(x.duration for x in v))
                 for k, v in per.items()]
        tot = [p.total for p in self.samples]
        return ProfileStats(self.samples[-1].source, self.g.structural_hash(), len(self.samples),
                            min(tot), sum(tot) / len(tot), nodes)

    # timing trends (same collect -> flush -> trend cycle as metric observation)
    def collect_timings(self, tags: Sequence[str]) -> None:
        if not self.samples:
            return
        for t in tags:
            self._collected.setdefault(t, []).append(self.samples[-1].timing(t))

    def flush_timings(self, tags: Sequence[str] = ()) -> None:
        for t in (tags or list(self._collected)):
            v = self._collected.pop(t, [])
            if v:
                self._history.setdefault(t, []).append(sum(v) / len(v))

    def timing_trend(self, tag: str):
        from .trend import Trend
        return Trend(list(self._history.get(tag, [])))

    def reset_timing_trend(self, tags: Sequence[str]) -> None:
        for t in tags:
            self._history.pop(t, None)


# ----------------------------------------------------------------- heatmap
def _heat(f: float) -> str:
    """White -> red by fraction of the slowest node's time."""
    f = max(0.0, min(1.0, f))
    g = int(255 * (1 - f))
    return f"rgb(255,{g},{g})"


def heatmap_svg(graph, profile: Optional[Profile] = None, path: Optional[str] = None) -> str:
    """Self-contained SVG: one row per execution level, one box per node,
    filled by its share of the slowest node's time (no graphviz needed)."""
    prof = profile or (graph.profile() if hasattr(graph, "profile") else None)
    dur = {n.id: n.duration for n in prof.nodes} if prof else {}
    tmax = max(dur.values()) if dur else 0.0
    bw, bh, gap = 170, 44, 16
    width = max(len(l) for l in graph.levels) * (bw + gap) + gap
    height = len(graph.levels) * (bh + gap) + gap + 24
    pos = {}
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" '
           f'font-family="monospace" font-size="11">']
    for li, lvl in enumerate(graph.levels):
        for j, ni in enumerate(lvl):
            x, y = gap + j * (bw + gap), gap + li * (bh + gap)
            pos[graph._node_list[ni].id] = (x + bw / 2, y, y + bh)
    for e in graph.edges:
        if e.from_node in pos and e.to_node in pos:
            (x1, _, y1), (x2, y2, _) = pos[e.from_node], pos[e.to_node]
            out.append(f'<line x1="{x1}" y1="{y1}" x2="{x2}" y2="{y2}" stroke="#888"/>')
    for li, lvl in enumerate(graph.levels):
        for j, ni in enumerate(lvl):
            n = graph._node_list[ni]
            x, y = gap + j * (bw + gap), gap + li * (bh + gap)
            d = dur.get(n.id)
            fill = _heat(d / tmax) if d is not None and tmax > 0 else "#eee"
            label = html.escape(n.id[:22])
            ms = f"{d * 1e3:.3f} ms" if d is not None else "-"
            out.append(f'<rect x="{x}" y="{y}" width="{bw}" height="{bh}" rx="4" fill="{fill}" '
                       f'stroke="#333"><title>{label}: {ms}</title></rect>')
            out.append(f'<text x="{x + 6}" y="{y + 17}">{label}</text>')
            out.append(f'<text x="{x + 6}" y="{y + 33}">{ms}</text>')
    total = f"total {prof.total * 1e3:.3f} ms ({prof.source})" if prof else "no profile"
    out.append(f'<text x="{gap}" y="{height - 8}">{html.escape(total)}</text></svg>')
    svg = "\n".join(out)
    if path:
        with open(path, "w") as f:
            f.write(svg)
    return svg


# ----------------------------------------------------------------- plots and logs
def format_duration(secs: float) -> str:
    if secs < 60:
        return f"{secs:.1f}s"
    m, s = divmod(int(secs), 60)
    if m < 60:
        return f"{m}m{s:02d}s"
    h, m = divmod(m, 60)
    return f"{h}h{m:02d}m"


def _plot_html(series: Dict[str, List[float]], title: str) -> str:
    data = json.dumps(series)
    return f"""<!doctype html><html><head><meta charset="utf-8"><title>{html.escape(title)}</title>
</head><body><h3>{html.escape(title)}</h3><div id="p"></div><script>
const S = {data}, NS = 'http://www.w3.org/2000/svg', W = 520, H = 140;
for (const [k, ys] of Object.entries(S)) {{
  if (!ys.length) continue;
  const mn = Math.min(...ys), mx = Math.max(...ys), sp = (mx - mn) || 1;
  const svg = document.createElementNS(NS, 'svg'); svg.setAttribute('width', W); svg.setAttribute('height', H + 22);
  const pl = document.createElementNS(NS, 'polyline');
  pl.setAttribute('points', ys.map((y, i) => `${{i / Math.max(ys.length - 1, 1) * W}},${{H - (y - mn) / sp * H}}`).join(' '));
  pl.setAttribute('fill', 'none'); pl.setAttribute('stroke', 'steelblue'); svg.appendChild(pl);
  const t = document.createElementNS(NS, 'text'); t.setAttribute('y', H + 16);
  t.textContent = `${{k}}  last=${{ys[ys.length - 1].toPrecision(4)}}  min=${{mn.toPrecision(4)}}  max=${{mx.toPrecision(4)}}`;
  svg.appendChild(t); document.getElementById('p').appendChild(svg);
}}
</script></body></html>"""


def plot_html(graph, path: str, tags: Sequence[str] = ()) -> None:
    keys = list(tags) or sorted(graph._history)
    with open(path, "w") as f:
        f.write(_plot_html({k: graph._history.get(k, []) for k in keys}, "metric trends"))


def plot_timings_html(graph, path: str, tags: Sequence[str] = ()) -> None:
    p = graph.profiler
    keys = list(tags) or sorted(p._history)
    with open(path, "w") as f:
        f.write(_plot_html({k: p._history.get(k, []) for k in keys}, "node timing trends (s)"))


def _export(hist: Dict[str, List[float]], path: str, tags: Sequence[str]) -> None:
    keys = list(tags) or sorted(hist)
    n = max((len(hist.get(k, [])) for k in keys), default=0)
    with open(path, "w") as f:
        f.write(",".join(["flush"] + keys) + "\n")
        for i in range(n):
            row = [str(i)] + [repr(hist[k][i]) if i < len(hist.get(k, [])) else "" for k in keys]
            f.write(",".join(row) + "\n")


def export_trends(graph, path: str, tags: Sequence[str] = ()) -> None:
    _export(graph._history, path, tags)


def export_timing_trends(graph, path: str, tags: Sequence[str] = ()) -> None:
    _export(graph.profiler._history, path, tags)


def write_log(graph, path: str, total_epochs: int, tags: Sequence[str] = ()) -> None:
    """Plain-text training log: one line per flush with the tags' values."""
    keys = list(tags) or sorted(graph._history)
    n = max((len(graph._history.get(k, [])) for k in keys), default=0)
    with open(path, "w") as f:
        for i in range(n):
            vals = " ".join(f"{k}={graph._history[k][i]:.5g}" for k in keys
                            if i < len(graph._history.get(k, [])))
            f.write(f"epoch {i + 1}/{total_epochs} {vals}\n")


# ----------------------------------------------------------------- snapshots
class ModelSnapshot:
    """CPU copy of a model's named parameters and buffers, taken at one
    instant (device-to-host copies into pinned memory on a side stream), so the
    model can keep training while the snapshot is written."""

    def __init__(self, named: List[Tuple[str, torch.Tensor]], structural_hash: Optional[str] = None,
                 event=None):
        self.named = named
        self.structural_hash = structural_hash
        self._event = event

    @staticmethod
    def take(module, structural_hash: Optional[str] = None) -> "ModelSnapshot":
        if hasattr(module, "graph_named_parameters"):  # graph names: tags and node ids
            items = list(module.graph_named_parameters()) + list(module.graph_named_buffers())
        else:
            items = list(module.named_parameters()) + list(module.named_buffers())
        cuda = any(t.is_cuda for _, t in items)
        out, ev = [], None
        if cuda:
            cur = torch.cuda.current_stream()
            side = torch.cuda.Stream()
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                for n, t in items:
                    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                    h.copy_(t.detach(), non_blocking=True)
                    out.append((n, h))
                ev = torch.cuda.Event()
                ev.record(side)
        else:
            out = [(n, t.detach().clone()) for n, t in items]
        return ModelSnapshot(out, structural_hash, ev)

    def wait(self) -> None:
        if self._event is not None:
            self._event.synchronize()
            self._event = None

    def save_file(self, path: str) -> None:
        from ..nn.checkpoint import save_checkpoint
        self.wait()
        save_checkpoint(path, self.named, (), self.structural_hash)

    def save_background(self, path: str) -> threading.Thread:
        """Write on a detached thread; join the returned thread to wait."""
        t = threading.Thread(target=self.save_file, args=(path,), daemon=True)
        t.start()
        return t
