"""Training monitor (flodl/src/monitor/mod.rs:215-1030, timeline.rs, record.rs).

* ``Monitor``: per-epoch log line with ETA, metric history, resource sampling
  (CPU/RAM from /proc, GPU utilisation/memory through NVML when present),
  ``export_csv``, ``save_html`` (a self-contained HTML report) and a JSONL
  record log.
* ``Timeline``: a background sampler of resource use plus discrete events
  (syncs, anchor changes, epoch starts), saved as JSON/CSV.
* ``serve(port)``: a live dashboard over HTTP. ``/events`` is the whole-run
  epoch feed (Server-Sent Events, late-join backfill) and ``/history`` its
  JSON; with ``?path=`` the path-scoped record plane answers instead:
  ``/paths`` (known nodes), ``/node?path=p`` (latest record of ``p`` and its
  direct children), ``/history?path=p&n=N`` and ``/stream?path=p`` (SSE),
  backed by :class:`~flodl_b200.monitor.records.RecordStore`.
"""
from __future__ import annotations

import csv
import http.server
import json
import os
import queue
import socketserver
import threading
import time
from typing import Dict, List, Optional
from urllib.parse import parse_qs, urlparse

from .records import Leaf, RecordLog, RecordStore, build_tree, event_record


def _cpu_ram():
    try:
        with open("/proc/meminfo") as f:
            info = {ln.split(":")[0]: int(ln.split()[1]) for ln in f if ":" in ln}
        used = (info.get("MemTotal", 0) - info.get("MemAvailable", 0)) / 1024
        return {"ram_used_mb": used, "ram_total_mb": info.get("MemTotal", 0) / 1024}
    except OSError:
        return {}


def _gpu_stats():
    try:
        import pynvml  # nvidia-ml-py

        pynvml.nvmlInit()
        out = []
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            u = pynvml.nvmlDeviceGetUtilizationRates(h)
            m = pynvml.nvmlDeviceGetMemoryInfo(h)
            out.append({"gpu": i, "util": u.gpu, "mem_used_mb": m.used / 2 ** 20,
                        "mem_total_mb": m.total / 2 ** 20})
        return out
    except Exception:
        return []


class Monitor:
    def __init__(self, total_epochs: int, record_path: Optional[str] = None, quiet: bool = False,
                 record_dir: Optional[str] = None, records: Optional[RecordStore] = None):
        self.records = records or RecordStore(log=RecordLog(record_dir) if record_dir else None)
        self.total = total_epochs
        self.start = time.time()
        self.history: List[Dict] = []
        self.record_path = record_path
        self.quiet = quiet
        self._subscribers: List[queue.Queue] = []
        self._server = None

    def log(self, epoch: int, metrics: Dict[str, float], elapsed: Optional[float] = None) -> str:
        now = time.time()
        done = epoch + 1
        rate = (now - self.start) / done
        eta = rate * max(self.total - done, 0)
        rec = {"epoch": epoch, "time": now, "elapsed": now - self.start, "eta_s": eta, **metrics,
               **_cpu_ram()}
        self.history.append(rec)
        if self.record_path:
            with open(self.record_path, "a") as f:
                f.write(json.dumps(rec) + "\n")
        for q in list(self._subscribers):
            try:
                q.put_nowait(rec)
            except queue.Full:
                pass
        num = {k: float(v) for k, v in metrics.items() if isinstance(v, (int, float))}
        self.records.publish_tree(build_tree([Leaf([], 1.0, num)], epoch_complete=True), epoch=epoch)
        parts = " ".join(f"{k}={v:.4g}" if isinstance(v, float) else f"{k}={v}" for k, v in metrics.items())
        line = f"epoch {done}/{self.total} {parts} eta {eta:.0f}s"
        if not self.quiet:
            print(line, flush=True)
        return line

    def alert(self, message: str, sev: str = "warn", path: str = "root", **fields) -> None:
        """Alert lane: a ``log`` record delivered to every viewer at or above ``path``."""
        from .records import Severity
        self.records.publish(event_record(path, "log", message, Severity(sev), **fields))

    def export_csv(self, path: str) -> None:
        if not self.history:
            return
        keys = sorted({k for r in self.history for k in r})
        with open(path, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=keys)
            w.writeheader()
            w.writerows(self.history)

    def save_html(self, path: str, title: str = "flodl_b200 training") -> None:
        data = json.dumps(self.history)
        html = f"""<!doctype html><html><head><meta charset="utf-8"><title>{title}</title></head>
<body><h2>{title}</h2><div id="plots"></div><pre id="raw"></pre><script>
const H = {data};
const keys = [...new Set(H.flatMap(r => Object.keys(r)))].filter(k => !['epoch','time'].includes(k));
const svgNS = 'http://www.w3.org/2000/svg';
for (const k of keys) {{
  const ys = H.map(r => r[k]).filter(v => typeof v === 'number'); if (!ys.length) continue;
  const mn = Math.min(...ys), mx = Math.max(...ys) || 1, W = 480, Hh = 120;
  const svg = document.createElementNS(svgNS, 'svg'); svg.setAttribute('width', W); svg.setAttribute('height', Hh + 20);
  const pts = ys.map((y, i) => `${{(i / Math.max(ys.length - 1, 1)) * W}},${{Hh - (y - mn) / ((mx - mn) || 1) * Hh}}`).join(' ');
  const pl = document.createElementNS(svgNS, 'polyline'); pl.setAttribute('points', pts);
  pl.setAttribute('fill', 'none'); pl.setAttribute('stroke', 'steelblue'); svg.appendChild(pl);
  const t = document.createElementNS(svgNS, 'text'); t.setAttribute('y', Hh + 15); t.textContent = k; svg.appendChild(t);
  document.getElementById('plots').appendChild(svg);
}}
</script></body></html>"""
        with open(path, "w") as f:
            f.write(html)

    # ------------------------------------------------------------ live dashboard (SSE)
    def serve(self, port: int = 0) -> int:
        mon = self

        class H(http.server.BaseHTTPRequestHandler):
            def log_message(self, *a):
                pass

            def _json(self, obj, code=200):
                body = json.dumps(obj).encode()
                self.send_response(code)
                self.send_header("Content-Type", "application/json")
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def _sse(self, backfill, q, unsubscribe):
                self.send_response(200)
                self.send_header("Content-Type", "text/event-stream")
                self.send_header("Cache-Control", "no-cache")
                self.end_headers()
                try:
                    for rec in backfill:  # late-join backfill
                        self.wfile.write(f"data: {json.dumps(rec)}\n\n".encode())
                    self.wfile.flush()
                    while True:
                        try:
                            rec = q.get(timeout=15)
                        except queue.Empty:
                            self.wfile.write(b": keep-alive\n\n")
                            self.wfile.flush()
                            continue
                        self.wfile.write(f"data: {json.dumps(rec)}\n\n".encode())
                        self.wfile.flush()
                except Exception:
                    pass
                finally:
                    unsubscribe()

            def do_GET(self):
                url = urlparse(self.path)
                qs = parse_qs(url.query)
                p = qs.get("path", [None])[0]
                n = int(qs.get("n", ["256"])[0])
                if url.path == "/paths":
                    self._json(mon.records.paths())
                elif url.path == "/node":
                    self._json(mon.records.node(p or "root"))
                elif url.path == "/history":
                    self._json(mon.records.history(p, n) if p else mon.history)
                elif url.path == "/stream" and p:
                    q = mon.records.subscribe(p)
                    self._sse(mon.records.history(p, n), q, lambda: mon.records.unsubscribe(q))
                elif url.path in ("/stream", "/events"):
                    q: queue.Queue = queue.Queue(maxsize=1024)
                    mon._subscribers.append(q)
                    self._sse(list(mon.history), q, lambda: mon._subscribers.remove(q))
                else:
                    body = (b"<html><body>flodl_b200 monitor: /events /history /paths "
                            b"/node?path= /history?path= /stream?path=</body></html>")
                    self.send_response(200)
                    self.send_header("Content-Type", "text/html")
                    self.send_header("Content-Length", str(len(body)))
                    self.end_headers()
                    self.wfile.write(body)

        class S(socketserver.ThreadingMixIn, http.server.HTTPServer):
            daemon_threads = True

        srv = S(("127.0.0.1", port), H)
        self._server = srv
        threading.Thread(target=srv.serve_forever, daemon=True).start()
        return srv.server_address[1]

    def close(self) -> None:
        if self._server is not None:
            self._server.shutdown()
            self._server = None


class Timeline:
    """Background resource sampler with discrete events."""

    def __init__(self, interval_s: float = 0.1):
        self.interval = interval_s
        self.samples: List[Dict] = []
        self.events: List[Dict] = []
        self._stop = threading.Event()
        self._t: Optional[threading.Thread] = None

    def start(self):
        def run():
            while not self._stop.is_set():
                self.samples.append({"t": time.time(), **_cpu_ram(), "gpus": _gpu_stats()})
                self._stop.wait(self.interval)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        return self

    def event(self, kind: str, **fields) -> None:
        self.events.append({"t": time.time(), "kind": kind, **fields})

    def stop(self) -> None:
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)

    def save_json(self, path: str) -> None:
        with open(path, "w") as f:
            json.dump({"samples": self.samples, "events": self.events}, f)

    def save_html(self, path: str, title: str = "timeline") -> None:
        """Self-contained page: GPU utilisation and host RAM over time, with the
        discrete events (syncs, anchor changes, epochs) listed beneath."""
        import html as _html
        from ..ddp_report import line_chart_svg
        series = {}
        for smp in self.samples:
            for g in smp.get("gpus", []):
                series.setdefault(f"gpu{g['gpu']} util %", []).append(float(g.get("util", 0)))
            if "ram_used_mb" in smp:
                series.setdefault("host RAM used (GB)", []).append(smp["ram_used_mb"] / 1024)
        t0 = self.samples[0]["t"] if self.samples else (self.events[0]["t"] if self.events else 0.0)
        rows = "".join(f"<tr><td>{e['t'] - t0:.3f}</td><td>{_html.escape(e['kind'])}</td>"
                       f"<td>{_html.escape(json.dumps({k: v for k, v in e.items() if k not in ('t', 'kind')}))}</td></tr>"
                       for e in self.events)
        charts = "".join(line_chart_svg({k: v}, k) for k, v in series.items()) or "<p>no samples</p>"
        with open(path, "w") as f:
            f.write(f"<!doctype html><html><head><meta charset='utf-8'><title>{_html.escape(title)}</title>"
                    f"</head><body><h2>{_html.escape(title)}</h2>{charts}<h3>events</h3>"
                    f"<table border=1><tr><th>t (s)</th><th>kind</th><th>detail</th></tr>{rows}</table>"
                    f"</body></html>")

    def save_csv(self, path: str) -> None:
        with open(path, "w", newline="") as f:
            w = csv.writer(f)
            w.writerow(["t", "kind", "detail"])
            for e in self.events:
                w.writerow([e["t"], e["kind"], json.dumps({k: v for k, v in e.items() if k not in ("t", "kind")})])
