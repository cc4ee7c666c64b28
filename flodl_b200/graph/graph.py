"""Graph: the executable form of a FlowBuilder flow (a Module itself, so graphs
nest into graph trees).

Reference: flodl/src/graph/graph.rs, execution.rs, tree.rs, observe.rs,
checkpoint.rs. The topology (Kahn levels, execution order, consumer counts) is
compiled by the native runtime; execution walks the compiled schedule with
Vec-indexed slots and frees each intermediate after its last consumer. Hot
training loops capture the whole step in a CUDA graph, so host dispatch cost
is paid once.

Naming: ``named_parameters()`` returns floDl's ``"<tag or node id>/<name>"``
keys (``"encoder/weight"``, ``"linear_2/bias"``), deduplicated by identity,
with ``_0``/``_1`` suffixes for repeated local names. ``structural_hash()`` is
a SHA-256 over node ids, module names, parameter/buffer names and shapes,
nested graph hashes and the edge list.
"""
from __future__ import annotations

import time
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .._ext import native
from ..nn.module import Module, walk_modules
from .flow import DEFAULT_INPUT, DEFAULT_OUTPUT, FlowBuilder, MergeOp, Node
from .trend import Trend, TrendGroup


_ADD = object()  # plan marker: a two-input add node


class Graph(Module):
    NAME = "graph"

    def __init__(self, fb: FlowBuilder):
        super().__init__()
        self._node_list: List[Node] = list(fb.nodes.values())
        self._index = {n.id: i for i, n in enumerate(self._node_list)}
        self._modules_list = torch.nn.ModuleList(
            [n.module if n.module is not None else torch.nn.Identity() for n in self._node_list])
        self.edges = list(fb.edges)
        self.inputs = list(fb.inputs)
        self.input_names = list(fb.input_names)
        self.output = fb.current[0]
        self.forward_refs = list(fb.forward_refs)
        self.tag_names = dict(fb.taps)
        self.tag_groups_map = dict(fb.tag_groups)
        self._label = fb._label
        self.internal_tags = set(fb.internal_tags)
        n = len(self._node_list)
        edge_idx = [(self._index[e.from_node], self._index[e.to_node]) for e in self.edges]
        levels, order, consumers = native().compile_levels(n, edge_idx)
        self.levels: List[List[int]] = [list(l) for l in levels]
        self.order: List[int] = list(order)
        self._consumers = list(consumers)
        # per-node input wiring: list of (port index, src node idx, src port)
        self._in_edges: List[List[Tuple[int, int, str]]] = [[] for _ in range(n)]
        for e in self.edges:
            di = self._index[e.to_node]
            pi = self._node_list[di].input_ports.index(e.to_port)
            self._in_edges[di].append((pi, self._index[e.from_node], e.from_port))
        self._input_node = {self._index[p.node_id]: k for k, p in enumerate(self.inputs)}
        self._fwd_ref_state: Dict[str, Optional[torch.Tensor]] = {r.name: None for r in self.forward_refs}
        self._fwd_ref_readers: Dict[int, List[Tuple[int, str]]] = {}
        for r in self.forward_refs:
            ri = self._index[r.reader_id]
            port = self._node_list[ri].input_ports.index(f"ref_{r.name}")
            self._fwd_ref_readers.setdefault(ri, []).append((port, r.name))
        self._fwd_ref_writers = {r.name: self._index[r.writer_id] for r in self.forward_refs}
        self._tag_values: Dict[str, torch.Tensor] = {}
        self._collected: Dict[str, List[float]] = {}
        self._history: Dict[str, List[float]] = {}
        self._flush_count = 0
        self._step_count = 0
        self._epoch_count = 0
        self._profiling = False
        self._profiler = None
        self._timings: Dict[str, float] = {}
        self._level_of = {ni: li for li, lvl in enumerate(self.levels) for ni in lvl}
        self._plan_cache = None
        self._hash: Optional[str] = None
        self._optimizer = None
        self._scheduler = None
        self._lr_scale = 1.0
        self._frozen: set = set()

    # ------------------------------------------------------------ execution
    def _plan(self):
        """Per-node execution records, built once: (node index, node, in-edge
        (port, src) pairs, forward-ref reader ports, input slot or -1, tags,
        direct module or None, level)."""
        tag_of: Dict[int, List[str]] = {}
        for t, ref in self.tag_names.items():
            tag_of.setdefault(self._index[ref.node_id], []).append(t)
        plan = []
        for ni in self.order:
            node = self._node_list[ni]
            direct = None
            if (node.kind in ("module", "loop", "gate", "switch", "map") and len(node.input_ports) == 1
                    and ni not in self._fwd_ref_readers):
                direct = node.module
            elif (node.kind == "add" and len(node.input_ports) == 2 and ni not in self._fwd_ref_readers
                  and len(self._in_edges[ni]) == 2 and ni not in self._input_node):
                direct = _ADD
            plan.append((ni, node, [(pi, si) for pi, si, _ in self._in_edges[ni]],
                         self._fwd_ref_readers.get(ni, ()), self._input_node.get(ni, -1),
                         tag_of.get(ni, ()), direct, self._level_of[ni]))
        self._plan_cache = plan
        self._out_idx = self._index[self.output.node_id]
        self._keep = set(self._fwd_ref_writers.values()) | {self._out_idx}
        return plan

    def forward(self, *inputs):
        if len(inputs) == 1 and isinstance(inputs[0], (list, tuple)):
            inputs = tuple(inputs[0])
        if len(inputs) != len(self.inputs):
            raise ValueError(f"graph expects {len(self.inputs)} inputs, got {len(inputs)}")
        plan = self._plan_cache if self._plan_cache is not None else self._plan()
        slots: List[Optional[torch.Tensor]] = [None] * len(self._node_list)
        remaining = list(self._consumers)
        keep = self._keep
        tag_values = self._tag_values
        prof = self.profiler if self._profiling else None
        if prof is not None:
            prof.begin()
        for ni, node, ins, ref_ports, in_slot, tags, direct, level in plan:
            mark = prof.node_start() if prof is not None else None
            if direct is _ADD:  # residual join of two slots
                out = slots[ins[0][1]] + slots[ins[1][1]]
            elif direct is not None:  # one input, no forward refs: call the module
                x = inputs[in_slot] if in_slot >= 0 else slots[ins[0][1]]
                out = direct(x)
            else:
                args: List[Optional[torch.Tensor]] = [None] * len(node.input_ports)
                if in_slot >= 0:
                    args[0] = inputs[in_slot]
                for pi, si in ins:
                    args[pi] = slots[si]
                for pi, name in ref_ports:
                    args[pi] = self._fwd_ref_state.get(name)
                out = self._run_node(node, args)
            if prof is not None:
                prof.node_end(ni, mark, level)
            slots[ni] = out
            for t in tags:
                tag_values[t] = out
            for _pi, si in ins:  # free intermediates whose consumers all ran
                remaining[si] -= 1
                if remaining[si] == 0 and si not in keep:
                    slots[si] = None
        for name, wi in self._fwd_ref_writers.items():
            self._fwd_ref_state[name] = tag_values.get(name)
        if prof is not None:
            p = prof.end()
            for n in p.nodes:
                self._timings[n.id] = self._timings.get(n.id, 0.0) + n.duration
        return slots[self._out_idx]

    def forward_multi(self, inputs: Sequence[torch.Tensor]):
        return self.forward(*inputs)

    @staticmethod
    def _run_node(node: Node, args):
        k = node.kind
        if k in ("module", "loop", "gate", "switch", "map"):
            x = args[0]
            refs = {}
            for port, v in zip(node.input_ports[1:], args[1:]):
                if port.startswith("ref_") and v is not None:
                    refs[port[4:]] = v
            if refs:
                m = node.module
                named = m.as_named_input() if hasattr(m, "as_named_input") else None
                if named is not None:
                    return named.forward_named(x, refs)
                for name in sorted(refs):
                    x = x + refs[name]
            return node.module(x)
        if k == "add":
            out = args[0]
            for a in args[1:]:
                out = out + a
            return out
        if k == "merge":
            out = args[0]
            for a in args[1:]:
                out = out + a
            if node.merge_op == MergeOp.MEAN:
                out = out / len(args)
            return out
        if k == "input":
            return args[0]
        raise RuntimeError(f"unknown node kind {k}")

    # ------------------------------------------------------------ state
    def reset_state(self) -> None:
        for k in self._fwd_ref_state:
            self._fwd_ref_state[k] = None
        for m in self._modules_list:
            if isinstance(m, Module):
                m.reset()

    def detach_state(self) -> None:
        for k, v in self._fwd_ref_state.items():
            if v is not None:
                self._fwd_ref_state[k] = v.detach()
        for m in self._modules_list:
            if isinstance(m, Module):
                m.detach_state()

    def has_state(self) -> bool:
        return any(v is not None for v in self._fwd_ref_state.values())

    def end_step(self) -> None:
        self._step_count += 1
        self.detach_state()

    def end_sequence(self) -> None:
        self.reset_state()

    def end_epoch(self) -> None:
        self._epoch_count += 1

    def step_count(self) -> int:
        return self._step_count

    def epoch_count(self) -> int:
        return self._epoch_count

    # ------------------------------------------------------------ naming
    def label(self) -> Optional[str]:
        return self._label

    def _prefix_of(self) -> Dict[int, str]:
        out: Dict[int, str] = {}
        for tag, ref in self.tag_names.items():
            out.setdefault(self._index[ref.node_id], tag)
        return out

    def _named_items(self, get) -> List[Tuple[str, torch.Tensor]]:
        pref = self._prefix_of()
        result = []
        seen = set()
        for ni in self.order:
            node = self._node_list[ni]
            if node.module is None:
                continue
            prefix = pref.get(ni, node.id)
            items = get(node.module)
            counts: Dict[str, int] = {}
            for name, _ in items:
                counts[name] = counts.get(name, 0) + 1
            idx: Dict[str, int] = {}
            for name, t in items:
                if id(t) in seen:
                    continue
                seen.add(id(t))
                if counts[name] > 1:
                    q = f"{prefix}/{name}_{idx.get(name, 0)}"
                    idx[name] = idx.get(name, 0) + 1
                else:
                    q = f"{prefix}/{name}"
                result.append((q, t))
        return result

    @staticmethod
    def _local_params(m):
        if isinstance(m, Graph):
            return m.graph_named_parameters()
        return [(n.replace(".", "/"), p) for n, p in torch.nn.Module.named_parameters(m)]

    @staticmethod
    def _local_buffers(m):
        if isinstance(m, Graph):
            return m.graph_named_buffers()
        return [(n.replace(".", "/"), b) for n, b in torch.nn.Module.named_buffers(m)]

    def graph_named_parameters(self) -> List[Tuple[str, torch.Tensor]]:
        return self._named_items(self._local_params)

    def graph_named_buffers(self) -> List[Tuple[str, torch.Tensor]]:
        return self._named_items(self._local_buffers)

    # floDl spelling returns the graph naming
    def named_parameters_flodl(self):
        return self.graph_named_parameters()

    # ------------------------------------------------------------ hashing
    def structural_hash(self) -> str:
        if self._hash is None:
            h = native().Sha256()
            for ni in self.order:
                node = self._node_list[ni]
                h.update_str(node.id)
                h.update(b"\0")
                m = node.module
                if m is not None:
                    name = m.name() if hasattr(m, "name") and callable(m.name) else type(m).__name__
                    h.update_str(name)
                    h.update(b"\0")
                    for tag, items in ((b"P", self._local_params(m)), (b"B", self._local_buffers(m))):
                        for pname, t in sorted(items, key=lambda kv: kv[0]):
                            h.update(tag)
                            h.update_str(pname)
                            h.update(b"\0")
                            for d in t.shape:
                                h.update_i64(int(d))
                    if isinstance(m, Graph):
                        h.update(b"G")
                        h.update_str(m.structural_hash())
            h.update_str("EDGES")
            for e in self.edges:
                for s in (e.from_node, e.from_port, e.to_node, e.to_port):
                    h.update_str(s)
                    h.update(b"\0")
            # tags by name: (node index, output-port index; every node has the
            # single output port), then the exposed input and output ports
            h.update_str("TAGS")
            for name in sorted(self.tag_names):
                ref = self.tag_names[name]
                h.update_str(name)
                h.update(b"\0")
                h.update_i64(self._index[ref.node_id])
                h.update_i64(0)
            h.update_str("INPUTS")
            for name, ref in zip(self.input_names, self.inputs):
                for s in (name, ref.node_id, ref.port):
                    h.update_str(s)
                    h.update(b"\0")
            h.update_str("OUTPUTS")
            for s in ("output", self.output.node_id, self.output.port):
                h.update_str(s)
                h.update(b"\0")
            self._hash = h.hexdigest()
        return self._hash

    def short_hash(self) -> str:
        return self.structural_hash()[:8]

    # ------------------------------------------------------------ observation
    def tagged(self, tag: str) -> Optional[torch.Tensor]:
        return self._tag_values.get(tag)

    def tag_names_list(self) -> List[str]:
        return sorted(self.tag_names)

    def tag_group(self, name: str) -> Optional[List[str]]:
        return self.tag_groups_map.get(name)

    def _expand(self, tags):
        out = []
        for t in tags:
            out.extend(self.tag_groups_map.get(t, [t]))
        return out

    def collect(self, tags: Sequence[str], reduce: str = "mean") -> None:
        for t in self._expand(tags):
            v = self._tag_values.get(t)
            if v is None:
                continue
            v = v.detach().float()
            x = float(v.mean() if reduce == "mean" else v.sum() if reduce == "sum" else v.max()
                      if reduce == "max" else v.min() if reduce == "min" else v.norm())
            self._collected.setdefault(t, []).append(x)

    def collect_with(self, tags, reduce: str):
        self.collect(tags, reduce)

    def record(self, tag: str, values: Sequence[float]) -> None:
        self._collected.setdefault(tag, []).extend(float(v) for v in values)

    def record_scalar(self, tag: str, value: float) -> None:
        self._collected.setdefault(tag, []).append(float(value))

    def collected(self, tag: str) -> List[float]:
        return list(self._collected.get(tag, []))

    def flush(self, tags: Sequence[str] = ()) -> None:
        keys = self._expand(tags) if tags else list(self._collected)
        for t in keys:
            vals = self._collected.pop(t, [])
            if vals:
                self._history.setdefault(t, []).append(sum(vals) / len(vals))
        self._flush_count += 1

    def flush_count(self) -> int:
        return self._flush_count

    def trend(self, tag: str) -> Trend:
        return Trend(list(self._history.get(tag, [])))

    def trends(self, tags: Sequence[str]) -> TrendGroup:
        return TrendGroup([self.trend(t) for t in self._expand(tags)])

    def reset_trend(self, tags: Sequence[str]) -> None:
        for t in self._expand(tags):
            self._history.pop(t, None)

    def latest_metrics(self) -> List[Tuple[str, float]]:
        return [(t, v[-1]) for t, v in sorted(self._history.items()) if v]

    def traces(self, name: str) -> Optional[List[torch.Tensor]]:
        ref = self.tag_names.get(name)
        node = self._node_list[self._index[ref.node_id]] if ref else self._node_by_id(name)
        if node is None or node.kind != "loop":
            return None
        return list(node.module.traces)

    def traces_by_node(self, node_id: str):
        n = self._node_by_id(node_id)
        return list(n.module.traces) if n is not None and n.kind == "loop" else None

    def last_trace(self, tag: str):
        tr = self.traces(tag)
        return tr[-1] if tr else None

    def _node_by_id(self, nid: str) -> Optional[Node]:
        i = self._index.get(nid)
        return self._node_list[i] if i is not None else None

    # ------------------------------------------------------------ graph tree
    def tree_children(self) -> Dict[str, "Graph"]:
        out = {}
        for n in self._node_list:
            if isinstance(n.module, Graph) and n.module.label():
                out[n.module.label()] = n.module
        return out

    def child_graph(self, label: str) -> Optional["Graph"]:
        return self.tree_children().get(label)

    def is_composed(self) -> bool:
        return bool(self.tree_children())

    def _resolve(self, path: str):
        """Resolve a dotted label path to (graph, tag-or-None)."""
        parts = path.split(".") if path else []
        g: Graph = self
        for i, p in enumerate(parts):
            child = g.child_graph(p)
            if child is not None:
                g = child
                continue
            if i == len(parts) - 1 and p in g.tag_names:
                if g is not self and p in g.internal_tags:
                    raise KeyError(f"tag {p!r} is internal to its graph")
                return g, p
            raise KeyError(f"unknown path component {p!r} in {path!r}")
        return g, None

    def validate_path(self, path: str) -> str:
        g, tag = self._resolve(path)
        return "tag" if tag is not None else "graph"

    def subgraph(self, path: str) -> "Graph":
        g, tag = self._resolve(path)
        if tag is not None:
            raise KeyError(f"{path!r} names a tag, not a subgraph")
        return g

    def _modules_at(self, path: str) -> List[torch.nn.Module]:
        g, tag = self._resolve(path)
        if tag is None:
            return [g]
        ni = g._index[g.tag_names[tag].node_id]
        return [g._node_list[ni].module] if g._node_list[ni].module is not None else []

    def parameters_at(self, path: str) -> List[torch.Tensor]:
        out, seen = [], set()
        for m in self._modules_at(path):
            for p in m.parameters():
                if id(p) not in seen:
                    seen.add(id(p))
                    out.append(p)
        return out

    def named_parameters_at(self, path: str):
        g, tag = self._resolve(path)
        items = g.graph_named_parameters()
        if tag is None:
            return items
        return [(n, p) for n, p in items if n.startswith(tag + "/")]

    def named_buffers_at(self, path: str):
        g, tag = self._resolve(path)
        items = g.graph_named_buffers()
        if tag is None:
            return items
        return [(n, b) for n, b in items if n.startswith(tag + "/")]

    def freeze(self, path: str) -> None:
        for p in self.parameters_at(path):
            p.requires_grad_(False)
        self._frozen.add(path)

    def thaw(self, path: str) -> None:
        for p in self.parameters_at(path):
            p.requires_grad_(True)
        self._frozen.discard(path)

    def is_frozen(self, path: str) -> bool:
        ps = self.parameters_at(path)
        return bool(ps) and all(not p.requires_grad for p in ps)

    def set_training_at(self, path: str, training: bool) -> None:
        for m in self._modules_at(path):
            m.train(training)

    def tagged_at(self, path: str):
        g, tag = self._resolve(path)
        return g.tagged(tag) if tag else None

    def collect_at(self, paths: Sequence[str]) -> None:
        for p in paths:
            g, tag = self._resolve(p)
            if tag:
                g.collect([tag])

    def record_at(self, path: str, value: float) -> None:
        g, tag = self._resolve(path)
        g.record_scalar(tag or path, value)

    def trend_at(self, path: str) -> Trend:
        g, tag = self._resolve(path)
        return g.trend(tag or path)

    def load_subgraph_checkpoint(self, path: str, file: str):
        from ..nn.checkpoint import load_checkpoint

        g = self.subgraph(path)
        return load_checkpoint(file, g.graph_named_parameters(), g.graph_named_buffers(),
                               g.structural_hash())

    # ------------------------------------------------------------ training glue
    def set_optimizer(self, optimizer) -> None:
        self._optimizer = optimizer

    def set_scheduler(self, scheduler) -> None:
        self._scheduler = scheduler

    def set_lr_scale(self, s: float) -> None:
        self._lr_scale = s

    def set_data_loader(self, loader) -> None:
        """Bind a streaming DataLoader: its prefetch sizing keeps ~3x the
        parameter bytes free for gradients and optimizer state (the step
        memory a VRAM probe cannot see before the first step)."""
        self._data_loader = loader
        if getattr(loader, "step_reserve_", None) is None:
            loader.step_reserve_ = 3 * sum(p.numel() * p.element_size() for p in self.parameters())

    def epoch_batches(self, epoch: int):
        """Batches of the bound loader for ``epoch``."""
        if getattr(self, "_data_loader", None) is None:
            raise RuntimeError("Graph.epoch_batches(): no data loader set")
        return self._data_loader.epoch(epoch)

    def step(self) -> None:
        """Optimizer step + scheduler update + zero_grad (graph/distributed.rs)."""
        if self._optimizer is None:
            raise RuntimeError("Graph.step(): no optimizer set")
        if self._scheduler is not None:
            self._optimizer.set_lr(self._scheduler.lr(self._step_count) * self._lr_scale)
        self._optimizer.step()
        self._optimizer.zero_grad()
        self.end_step()

    # ------------------------------------------------------------ profiling / viz
    def enable_profiling(self, on: bool = True) -> None:
        """Time every node of every forward with reusable device events (host
        clock on CPU); durations resolve once per forward."""
        self._profiling = on

    def disable_profiling(self) -> None:
        self._profiling = False

    def profiling(self) -> bool:
        return self._profiling

    @property
    def profiler(self):
        if self._profiler is None:
            from .profile import GraphProfiler
            self._profiler = GraphProfiler(self)
        return self._profiler

    def profile(self):
        """The last forward's :class:`~flodl_b200.graph.profile.Profile`, or None."""
        s = self.profiler.samples
        return s[-1] if s else None

    def profile_stats(self):
        return self.profiler.stats()

    def timing(self, tag: Optional[str] = None):
        """Accumulated seconds per node id, or the last forward's time of one tag."""
        if tag is None:
            return dict(self._timings)
        p = self.profile()
        return p.timing(tag) if p else 0.0

    def collect_timings(self, tags: Sequence[str]) -> None:
        self.profiler.collect_timings(tags)

    def flush_timings(self, tags: Sequence[str] = ()) -> None:
        self.profiler.flush_timings(tags)

    def timing_trend(self, tag: str) -> Trend:
        return self.profiler.timing_trend(tag)

    def reset_timing_trend(self, tags: Sequence[str]) -> None:
        self.profiler.reset_timing_trend(tags)

    def heatmap_svg(self, path: Optional[str] = None) -> str:
        from .profile import heatmap_svg
        return heatmap_svg(self, self.profile(), path)

    def plot_html(self, path: str, tags: Sequence[str] = ()) -> None:
        from .profile import plot_html
        plot_html(self, path, tags)

    def plot_timings_html(self, path: str, tags: Sequence[str] = ()) -> None:
        from .profile import plot_timings_html
        plot_timings_html(self, path, tags)

    def export_trends(self, path: str, tags: Sequence[str] = ()) -> None:
        from .profile import export_trends
        export_trends(self, path, tags)

    def export_timing_trends(self, path: str, tags: Sequence[str] = ()) -> None:
        from .profile import export_timing_trends
        export_timing_trends(self, path, tags)

    def write_log(self, path: str, total_epochs: int, tags: Sequence[str] = ()) -> None:
        from .profile import write_log
        write_log(self, path, total_epochs, tags)

    def snapshot_cpu(self):
        """A :class:`~flodl_b200.graph.profile.ModelSnapshot` for a background save."""
        from .profile import ModelSnapshot
        return ModelSnapshot.take(self, self.structural_hash())

    def describe(self) -> str:
        lines = [f"Graph {self._label or ''} [{self.short_hash()}] "
                 f"{len(self._node_list)} nodes, {len(self.levels)} levels, "
                 f"{sum(p.numel() for p in self.parameters())} params"]
        pref = self._prefix_of()
        for li, lvl in enumerate(self.levels):
            for ni in lvl:
                n = self._node_list[ni]
                tag = f" #{pref[ni]}" if ni in pref else ""
                lines.append(f"  L{li} {n.id} ({n.kind}){tag}")
        return "\n".join(lines)

    def dot(self) -> str:
        from .dot import graph_to_dot

        return graph_to_dot(self)

    def svg(self, path: Optional[str] = None) -> str:
        from .dot import render_svg

        return render_svg(self.dot(), path)
