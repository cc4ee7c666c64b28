"""Reports over DDP-bench results: comparison tables, ElChe detail, SVG charts.

Reference role: ddp-bench/src/report/{tables.rs, elche.rs, charts.rs} and the
post-hoc analysis of ddp-bench/src/analyze. Input is the list of JSON records
``flodl_b200.ddp_bench.run`` returns (one per model and mode); output is a
markdown report and hand-written SVG charts (no plotting dependency).

Tables: per model, each mode's wall time, samples/s, speed ratio against the
``solo`` run, first/final loss and loss ratio against solo, averaging rounds.
ElChe detail: the anchor (largest per-rank count) of each averaging window and
the per-rank batch-count ranges.
"""
from __future__ import annotations

import html
import json
from typing import Dict, List, Optional


def _by_model(results: List[dict]) -> Dict[str, Dict[str, dict]]:
    out: Dict[str, Dict[str, dict]] = {}
    for r in results:
        out.setdefault(r["model"], {})[r["mode"]] = r
    return out


def _fmt(v, p=4):
    if v is None:
        return "-"
    if isinstance(v, float):
        return f"{v:.{p}g}"
    return str(v)


def comparison_table(results: List[dict]) -> str:
    lines = []
    for model, modes in _by_model(results).items():
        solo = modes.get("solo")
        lines.append(f"### {model}\n")
        lines.append("| mode | ranks | wall s | samples/s | speed vs solo | first loss | final loss | "
                     "loss vs solo | averaging rounds |")
        lines.append("|---|---|---|---|---|---|---|---|---|")
        for mode, r in modes.items():
            sp = (r["samples_per_s"] / solo["samples_per_s"]) if solo and solo.get("samples_per_s") else None
            lr = ((r["final_loss"] / solo["final_loss"]) if solo and solo.get("final_loss")
                  and r.get("final_loss") is not None else None)
            lines.append(f"| {mode} | {len(r.get('devices', []))} | {_fmt(r.get('wall_s'))} | "
                         f"{_fmt(r.get('samples_per_s'))} | {_fmt(sp, 3)} | {_fmt(r.get('first_loss'))} | "
                         f"{_fmt(r.get('final_loss'))} | {_fmt(lr, 3)} | {r.get('syncs', '-')} |")
        lines.append("")
    return "\n".join(lines)


def elche_detail(results: List[dict]) -> str:
    lines = []
    for r in results:
        bc = r.get("batch_counts") or []
        if not bc:
            continue
        anchors = [max(c) for c in bc]
        ranks = len(bc[0])
        ranges = [f"{min(c[k] for c in bc)}-{max(c[k] for c in bc)}" for k in range(ranks)]
        lines.append(f"- **{r['model']} / {r['mode']}**: {len(bc)} windows; anchor sequence "
                     f"{anchors[:16]}{' ...' if len(anchors) > 16 else ''}; per-rank batches "
                     f"{', '.join(f'r{k} {v}' for k, v in enumerate(ranges))}")
    return "\n".join(lines) if lines else "_no cadence runs_"


def bar_chart_svg(values: Dict[str, float], title: str, unit: str = "", width: int = 520) -> str:
    """Horizontal bars, one per key, scaled to the largest value."""
    items = [(k, v) for k, v in values.items() if v is not None]
    h = 28 * len(items) + 40
    vmax = max((v for _, v in items), default=1.0) or 1.0
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{h}" '
           f'font-family="sans-serif" font-size="12">',
           f'<text x="8" y="18" font-weight="bold">{html.escape(title)}</text>']
    for i, (k, v) in enumerate(items):
        y = 30 + 28 * i
        w = (width - 220) * v / vmax
        out.append(f'<text x="8" y="{y + 15}">{html.escape(k)}</text>')
        out.append(f'<rect x="130" y="{y}" width="{w:.1f}" height="20" fill="steelblue"/>')
        out.append(f'<text x="{136 + w:.1f}" y="{y + 15}">{_fmt(v)} {html.escape(unit)}</text>')
    out.append("</svg>")
    return "\n".join(out)


def line_chart_svg(series: Dict[str, List[float]], title: str, width: int = 520, height: int = 200) -> str:
    colors = ["steelblue", "darkorange", "seagreen", "crimson", "purple", "gray"]
    pts = [v for s in series.values() for v in s]
    lo, hi = (min(pts), max(pts)) if pts else (0.0, 1.0)
    span = (hi - lo) or 1.0
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height + 40}" '
           f'font-family="sans-serif" font-size="12">',
           f'<text x="8" y="16" font-weight="bold">{html.escape(title)}</text>']
    for i, (name, s) in enumerate(series.items()):
        if not s:
            continue
        c = colors[i % len(colors)]
        xy = " ".join(f"{40 + (width - 60) * j / max(len(s) - 1, 1):.1f},"
                      f"{24 + height * (1 - (v - lo) / span):.1f}" for j, v in enumerate(s))
        out.append(f'<polyline points="{xy}" fill="none" stroke="{c}" stroke-width="1.5"/>')
        out.append(f'<text x="{40 + 110 * i}" y="{height + 36}" fill="{c}">{html.escape(name)}</text>')
    out.append("</svg>")
    return "\n".join(out)


def write_report(results: List[dict], path: str, charts_dir: Optional[str] = None) -> str:
    """Markdown report (and SVG charts beside it, linked from the report)."""
    import os
    parts = ["# DDP bench report\n", comparison_table(results), "## ElChe cadence\n", elche_detail(results), ""]
    if charts_dir:
        os.makedirs(charts_dir, exist_ok=True)
        for model, modes in _by_model(results).items():
            svg = bar_chart_svg({m: r.get("samples_per_s") for m, r in modes.items()},
                                f"{model}: throughput by mode", "samples/s")
            p = os.path.join(charts_dir, f"{model}-throughput.svg")
            with open(p, "w") as f:
                f.write(svg)
            parts.append(f"![{model} throughput]({os.path.relpath(p, os.path.dirname(path) or '.')})\n")
    text = "\n".join(parts)
    with open(path, "w") as f:
        f.write(text)
    return text


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="report over ddp_bench JSON lines")
    ap.add_argument("results", help="file with one ddp_bench JSON record per line")
    ap.add_argument("--out", default="ddp_report.md")
    ap.add_argument("--charts", default=None)
    a = ap.parse_args(argv)
    with open(a.results) as f:
        rs = [json.loads(l) for l in f if l.strip().startswith("{")]
    write_report(rs, a.out, a.charts)
    print(a.out)


if __name__ == "__main__":
    main()
