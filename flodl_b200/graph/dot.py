"""Graphviz DOT export of a Graph, optional SVG rendering through the ``dot``
CLI (flodl/src/graph/dot.rs), and a per-node timing heatmap."""
from __future__ import annotations

import shutil
import subprocess
from typing import Optional


def graph_to_dot(g) -> str:
    pref = g._prefix_of()
    timing = g.timing()
    tmax = max(timing.values()) if timing else 0.0
    lines = ["digraph flodl {", "  rankdir=TB;", '  node [shape=box, fontname="monospace"];']
    for i, n in enumerate(g._node_list):
        label = n.id + (f"\\n#{pref[i]}" if i in pref else "")
        if n.module is not None:
            np_ = sum(p.numel() for p in n.module.parameters())
            if np_:
                label += f"\\n{np_} params"
        color = ""
        if tmax > 0 and n.id in timing:
            heat = timing[n.id] / tmax
            color = f', style=filled, fillcolor="1.0 {heat:.2f} 1.0"'
        shape = "ellipse" if n.kind in ("add", "merge", "input") else "box"
        lines.append(f'  "{n.id}" [label="{label}", shape={shape}{color}];')
    for e in g.edges:
        attr = "" if e.to_port in ("input", "input_0", "input_1") else f' [label="{e.to_port}"]'
        lines.append(f'  "{e.from_node}" -> "{e.to_node}"{attr};')
    lines.append("}")
    return "\n".join(lines)


def render_svg(dot_src: str, path: Optional[str] = None) -> str:
    exe = shutil.which("dot")
    if exe is None:
        raise RuntimeError("graphviz `dot` is not installed; use Graph.dot() for the DOT source")
    out = subprocess.run([exe, "-Tsvg"], input=dot_src.encode(), capture_output=True, check=True).stdout.decode()
    if path:
        with open(path, "w") as f:
            f.write(out)
    return out
