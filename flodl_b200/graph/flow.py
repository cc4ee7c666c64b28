"""FlowBuilder: a fluent builder for computation graphs that reads as data flow.

Reference: flodl/src/graph/flow.rs:58-597. Builder methods never raise; the
first error is remembered and surfaces from :meth:`FlowBuilder.build`.

    g = (FlowBuilder.from_(Linear(4, 8)).through(GELU()).through(LayerNorm(8))
         .also(Linear(8, 8)).through(Linear(8, 2)).build())
    y = g(x)
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import torch

from ..nn.layers import Identity
from ..nn.module import Module

DEFAULT_INPUT = "input"
DEFAULT_OUTPUT = "output"


class MergeOp(enum.Enum):
    ADD = "add"
    MEAN = "mean"

    Add = "add"  # floDl spelling aliases
    Mean = "mean"


@dataclass
class NodeRef:
    node_id: str
    port: str = DEFAULT_OUTPUT


@dataclass
class Edge:
    from_node: str
    from_port: str
    to_node: str
    to_port: str


@dataclass
class Node:
    id: str
    kind: str  # module | add | merge | input | loop | gate | switch | map
    module: Optional[torch.nn.Module] = None
    input_ports: List[str] = field(default_factory=lambda: [DEFAULT_INPUT])
    merge_op: Optional[MergeOp] = None
    extra: dict = field(default_factory=dict)


@dataclass
class ForwardRef:
    name: str
    reader_id: str
    writer_id: str
    writer_port: str


class FlowBuilder:
    def __init__(self, module: Optional[torch.nn.Module] = None):
        self.nodes: Dict[str, Node] = {}
        self.edges: List[Edge] = []
        self.inputs: List[NodeRef] = []
        self.current: List[NodeRef] = []
        self.taps: Dict[str, NodeRef] = {}
        self.on_target: Optional[NodeRef] = None
        self.fork_target: Optional[NodeRef] = None
        self.counter = 0  # one sequence over every node kind: linear_1, gelu_2, linear_3
        self.input_names: List[str] = []
        self.err: Optional[str] = None
        self.pending: Dict[str, List[str]] = {}
        self.forward_refs: List[ForwardRef] = []
        self.tag_groups: Dict[str, List[str]] = {}
        self._label: Optional[str] = None
        self.internal_tags = set()
        self._verbose = False
        ref = self._add_module(module if module is not None else Identity())
        self.inputs.append(NodeRef(ref.node_id, DEFAULT_INPUT))
        self.input_names.append(DEFAULT_INPUT)
        self.on_target = ref
        self.current = [ref]

    # floDl's constructor names
    @classmethod
    def from_(cls, module: torch.nn.Module) -> "FlowBuilder":
        return cls(module)

    @classmethod
    def new(cls) -> "FlowBuilder":
        return cls(Identity())

    # ------------------------------------------------------------ internals
    def fail(self, msg: str) -> None:
        if self.err is None:
            self.err = msg

    def next_id(self, prefix: str) -> str:
        """Node ids as the reference's builder forms them: the prefix and one
        counter shared by every node of the graph (flodl/src/graph/flow.rs
        ``next_id``), so untagged parameters get the same checkpoint keys."""
        self.counter += 1
        return f"{prefix}_{self.counter}"

    def _add_node(self, node: Node) -> NodeRef:
        self.nodes[node.id] = node
        return NodeRef(node.id, DEFAULT_OUTPUT)

    def _add_module(self, module: torch.nn.Module) -> NodeRef:
        name = module.name() if hasattr(module, "name") and callable(module.name) else type(module).__name__.lower()
        return self._add_node(Node(self.next_id(name), "module", module))

    def _edge(self, src: NodeRef, dst_id: str, port: str = DEFAULT_INPUT) -> None:
        self.edges.append(Edge(src.node_id, src.port, dst_id, port))

    def _single(self, what: str) -> bool:
        if self.err is not None:
            return False
        if len(self.current) != 1:
            self.fail(f"{what} requires single stream")
            return False
        return True

    # ------------------------------------------------------------ metadata
    def label(self, name: str) -> "FlowBuilder":
        self._label = name
        return self

    def internal(self, tag: str) -> "FlowBuilder":
        self.internal_tags.add(tag)
        return self

    def verbose(self, enabled: bool = True) -> "FlowBuilder":
        self._verbose = enabled
        return self

    # ------------------------------------------------------------ sequential
    def through(self, module: torch.nn.Module) -> "FlowBuilder":
        if not self._single("through"):
            return self
        prev = self.current[0]
        ref = self._add_module(module)
        self._edge(prev, ref.node_id)
        self.on_target = ref
        self.current = [ref]
        return self

    def fork(self, module: torch.nn.Module) -> "FlowBuilder":
        """Side branch on the current stream; the main stream continues unchanged."""
        if not self._single("fork"):
            return self
        prev = self.current[0]
        ref = self._add_module(module)
        self._edge(prev, ref.node_id)
        self.on_target = ref
        self.fork_target = ref
        return self

    def also(self, module: torch.nn.Module) -> "FlowBuilder":
        """Residual: ``stream + module(stream)``."""
        if not self._single("also"):
            return self
        prev = self.current[0]
        mref = self._add_module(module)
        add = self._add_node(Node(self.next_id("add"), "add", input_ports=["input_0", "input_1"]))
        self._edge(prev, mref.node_id)
        self._edge(prev, add.node_id, "input_0")
        self._edge(mref, add.node_id, "input_1")
        self.on_target = mref
        self.current = [add]
        return self

    def also_with(self, skip: torch.nn.Module, main: torch.nn.Module) -> "FlowBuilder":
        """Residual with a transformed skip: ``skip(stream) + main(stream)``."""
        if not self._single("also_with"):
            return self
        prev = self.current[0]
        sref = self._add_module(skip)
        mref = self._add_module(main)
        add = self._add_node(Node(self.next_id("add"), "add", input_ports=["input_0", "input_1"]))
        self._edge(prev, sref.node_id)
        self._edge(prev, mref.node_id)
        self._edge(sref, add.node_id, "input_0")
        self._edge(mref, add.node_id, "input_1")
        self.on_target = mref
        self.current = [add]
        return self

    # ------------------------------------------------------------ tags
    def _resolve_pending(self, name: str, writer: NodeRef) -> None:
        for reader in self.pending.pop(name, []):
            self.forward_refs.append(ForwardRef(name, reader, writer.node_id, writer.port))

    def tag(self, name: str) -> "FlowBuilder":
        if not self._single("tag"):
            return self
        if name in self.taps:
            self.fail(f"duplicate tag: {name}")
            return self
        cur = self.fork_target if self.fork_target is not None else self.current[0]
        self.fork_target = None
        self.taps[name] = cur
        self._resolve_pending(name, cur)
        return self

    def tag_group(self, name: str) -> "FlowBuilder":
        if self.err is not None:
            return self
        if len(self.current) < 2:
            self.fail(f"tag_group({name!r}) requires multiple streams (got {len(self.current)}); "
                      "use tag for single-stream")
            return self
        if name in self.tag_groups:
            self.fail(f"duplicate tag group: {name!r}")
            return self
        if name in self.taps:
            self.fail(f"tag group {name!r} conflicts with existing tag")
            return self
        names = []
        for i, cur in enumerate(self.current):
            t = f"{name}_{i}"
            if t in self.taps:
                self.fail(f"tag_group({name!r}): suffixed name {t!r} conflicts with existing tag")
                return self
            self.taps[t] = cur
            names.append(t)
            self._resolve_pending(t, cur)
        self.tag_groups[name] = names
        return self

    def input(self, names: Sequence[str]) -> "FlowBuilder":
        """Named auxiliary graph inputs (forward takes them after the main input)."""
        if self.err is not None:
            return self
        for name in names:
            if name in self.taps:
                self.fail(f"input tag {name!r} conflicts with existing tag")
                return self
            ref = self._add_node(Node(self.next_id(f"input_{name}"), "input"))
            self.taps[name] = ref
            self.inputs.append(NodeRef(ref.node_id, DEFAULT_INPUT))
            self.input_names.append(name)
            self._resolve_pending(name, ref)
        return self

    def using(self, refs: Sequence[str]) -> "FlowBuilder":
        """Feed tagged outputs to the preceding module as named extra inputs.
        Refs tagged later are forward references (previous call's value)."""
        if self.err is not None or not refs:
            return self
        if self.on_target is not None:
            targets = [self.on_target]
        elif len(self.current) > 1:
            targets = list(self.current)
        else:
            self.fail("using requires a preceding through, split, or merge")
            return self
        for t in targets:
            node = self.nodes[t.node_id]
            for r in refs:
                port = f"ref_{r}"
                if port in node.input_ports:
                    self.fail(f"using: duplicate ref {r!r}")
                    return self
                node.input_ports.append(port)
                if r in self.taps:
                    self._edge(self.taps[r], node.id, port)
                else:
                    self.pending.setdefault(r, []).append(node.id)
        return self

    # ------------------------------------------------------------ branches
    def split(self, modules: Sequence[torch.nn.Module]) -> "FlowBuilder":
        if not self._single("split"):
            return self
        if len(modules) < 2:
            self.fail("split requires at least 2 branches")
            return self
        prev = self.current[0]
        branches = []
        for m in modules:
            ref = self._add_module(m)
            self._edge(prev, ref.node_id)
            branches.append(ref)
        self.on_target = None
        self.current = branches
        return self

    def merge(self, op: MergeOp = MergeOp.ADD) -> "FlowBuilder":
        if self.err is not None:
            return self
        if len(self.current) < 2:
            self.fail("merge requires multiple streams (after split)")
            return self
        op = MergeOp(op.value if isinstance(op, MergeOp) else op)
        n = len(self.current)
        ref = self._add_node(Node(self.next_id("merge"), "merge",
                                  input_ports=[f"input_{i}" for i in range(n)], merge_op=op))
        for i, b in enumerate(self.current):
            self._edge(b, ref.node_id, f"input_{i}")
        self.on_target = ref
        self.current = [ref]
        return self

    # ------------------------------------------------------------ control flow
    def loop_body(self, body: torch.nn.Module) -> "LoopBuilder":
        from .control import LoopBuilder

        return LoopBuilder(self, body)

    def switch(self, router: torch.nn.Module, branches: Sequence[torch.nn.Module]) -> "FlowBuilder":
        from .control import SwitchComposite

        return self._composite("switch", SwitchComposite(router, list(branches)),
                               min_branches=len(branches))

    def gate(self, router: torch.nn.Module, experts: Sequence[torch.nn.Module]) -> "FlowBuilder":
        from .control import GateComposite

        if len(experts) < 2:
            self.fail("gate requires at least 2 experts")
            return self
        return self._composite("gate", GateComposite(router, list(experts)))

    def map(self, body: torch.nn.Module) -> "MapBuilder":
        from .control import MapBuilder

        return MapBuilder(self, body)

    def _composite(self, prefix: str, module: torch.nn.Module, min_branches: int = 2,
                   source: Optional[NodeRef] = None) -> "FlowBuilder":
        if not self._single(prefix):
            return self
        if min_branches < 1:
            self.fail(f"{prefix} requires at least 1 branch")
            return self
        src = source if source is not None else self.current[0]
        ref = self._add_node(Node(self.next_id(prefix), prefix, module))
        self._edge(src, ref.node_id)
        self.current = [ref]
        self.on_target = ref
        return self

    # ------------------------------------------------------------ build
    def build(self):
        from .graph import Graph

        if self.err is not None:
            raise ValueError(self.err)
        if len(self.current) != 1:
            raise ValueError("build requires a single output stream (merge the split branches first)")
        if self.pending:
            raise ValueError(f"unresolved forward references: {sorted(self.pending)}")
        g = Graph(self)
        from ..utils import log
        if self._verbose or log.verbosity() >= log.Verbosity.VERBOSE:
            log.msg(g.describe()) if self._verbose else log.verbose(g.describe())
        return g
