"""Record plane: work-weighted tree, delivery predicate, bounded JSONL log,
live store over HTTP/SSE, dashboard sink (reference: monitor/record.rs,
record_log.rs, record_store.rs, server.rs tests)."""
import json
import os
import threading
import time
import urllib.request

import pytest

from flodl_b200.monitor.monitor import Monitor
from flodl_b200.monitor.records import (DashboardEmitter, DashboardSink, Leaf, RecordLog,
                                        RecordStore, Reduction, Severity, build_tree, delivers,
                                        event_record, rank_record_path)


def _leaves():
    return [Leaf(["hostA", "rank0"], 100, {"loss": 2.0, "throughput": 10.0, "acc": 0.5}, {"gpu_util": 80}),
            Leaf(["hostA", "rank1"], 300, {"loss": 1.0, "throughput": 30.0}, {"gpu_util": 40}),
            Leaf(["hostB", "rank2"], 0, {"loss": 9.0, "throughput": 0.0, "acc": 0.9}, {}),
            Leaf(["hostB", "rank3"], 100, {"loss": 4.0, "throughput": 10.0}, {"gpu_util": 60}, alive=False)]


def test_tree_is_work_weighted_and_hierarchical_equals_flat():
    t = build_tree(_leaves(), {"acc": Reduction.Max})
    assert [c.path_str for c in t.children] == ["root/hostA", "root/hostB"]
    a, b = t.children
    assert a.metrics["loss"] == pytest.approx((2 * 100 + 1 * 300) / 400)
    assert b.metrics["loss"] == pytest.approx(4.0)  # zero-work rank excluded from the mean
    flat = (2 * 100 + 1 * 300 + 4 * 100) / 500
    assert t.metrics["loss"] == pytest.approx(flat) and t.work == 500
    assert t.metrics["throughput"] == 50.0            # core key: sum
    assert t.metrics["acc"] == 0.9                    # user reduction: max
    assert "gpu_util" not in b.children[0].res        # absent, not zero
    assert a.res["gpu_util"] == pytest.approx((80 * 100 + 40 * 300) / 400)
    assert b.alive and not b.children[1].alive
    recs = t.flat_records(1.0, tick=3)
    assert recs[0]["path"] == "root" and recs[0]["children"] == 2 and len(recs) == 7
    assert rank_record_path(3, ["a", "a", "b", "b"]) == "root/b/rank3"
    assert rank_record_path(0, ["a"]) == "root" and rank_record_path(1, ["a", "a"]) == "root/rank1"


def test_delivery_predicate():
    node = lambda p: {"kind": "node", "path": p}
    assert delivers(node("root"), "root") and delivers(node("root/h"), "root")
    assert not delivers(node("root/h/rank0"), "root")       # metrics: depth 1
    assert delivers(event_record("root/h/rank0", "log", "oom", Severity.Critical), "root")  # alerts: any depth
    assert not delivers(node("root/hx"), "root/h")


def test_record_log_rotates_and_tails(tmp_path):
    log = RecordLog(str(tmp_path), segment_bytes=400, segments=3)
    for i in range(60):
        log.append({"kind": "node", "path": "root/h/rank0", "i": i})
    tail = log.tail("root/h/rank0", 5)
    assert [r["i"] for r in tail] == [55, 56, 57, 58, 59]
    files = list((tmp_path / "root" / "h").iterdir())
    assert len(files) == 3 and sum(f.stat().st_size for f in files) <= 3 * 400 + 100
    bad = RecordLog("/proc/flodl-cannot-write")
    bad.append({"path": "root"})  # swallowed, never raises


def test_store_and_http_record_plane():
    mon = Monitor(3, quiet=True)
    port = mon.serve(0)
    mon.records.publish_tree(build_tree(_leaves()), tick=1)
    base = f"http://127.0.0.1:{port}"
    paths = json.loads(urllib.request.urlopen(base + "/paths", timeout=5).read())
    assert "root/hostA/rank1" in paths
    nd = json.loads(urllib.request.urlopen(base + "/node?path=root/hostA", timeout=5).read())
    assert nd["node"]["path"] == "root/hostA" and len(nd["children"]) == 2
    got = []

    def listen():
        r = urllib.request.urlopen(base + "/stream?path=root&n=0", timeout=10)
        for line in r:
            if line.startswith(b"data: "):
                got.append(json.loads(line[6:]))
                if len(got) >= 2:
                    return

    th = threading.Thread(target=listen, daemon=True)
    th.start()
    time.sleep(0.5)
    mon.alert("rank3 stalled", "critical", path="root/hostB/rank3")
    mon.records.publish({"kind": "node", "path": "root/hostB/rank3", "work": 1})  # depth 2: not delivered
    mon.log(0, {"loss": 1.5})
    th.join(10)
    assert [g["kind"] for g in got] == ["log", "node"] and got[1]["path"] == "root"
    hist = json.loads(urllib.request.urlopen(base + "/history?path=root&n=50", timeout=5).read())
    assert any(r.get("message") == "rank3 stalled" for r in hist)
    assert json.loads(urllib.request.urlopen(base + "/history", timeout=5).read())[0]["loss"] == 1.5
    mon.close()


def test_dashboard_sink_receives_signed_rank_records():
    store = RecordStore()
    key = b"d" * 16
    sink = DashboardSink(store, key)
    em = DashboardEmitter("127.0.0.1", sink.port, key)
    em.emit([{"kind": "node", "path": "root/rank0", "metrics": {"loss": 1.0}, "work": 64}])
    end = time.time() + 5
    while time.time() < end and "root/rank0" not in store.paths():
        time.sleep(0.02)
    assert store.node("root")["children"][0]["metrics"]["loss"] == 1.0
    bad = DashboardEmitter("127.0.0.1", sink.port, b"wrong-key-000000")
    bad.emit({"kind": "node", "path": "root/evil"})
    end = time.time() + 5
    while time.time() < end and sink.rejected == 0:
        time.sleep(0.02)
    assert sink.rejected == 1 and "root/evil" not in store.paths()
    em.close(), bad.close(), sink.close()


def test_timeline_spill_and_shipper_mirror_with_rotation(tmp_path):
    from flodl_b200.monitor.telemetry import TelemetryShipper, TimelineSpill, telemetry_dir
    d = telemetry_dir("job", str(tmp_path / "local"))
    assert os.path.basename(d).startswith("job-")
    spill = TimelineSpill(d, segment_bytes=600, flush_s=0.05)
    ship = TelemetryShipper(d, str(tmp_path / "shared"), interval_s=0.05)
    for i in range(60):
        spill.event("step", i=i)
        if i % 7 == 0:
            time.sleep(0.06)
    spill.close()
    assert ship.finish(10)
    lines = (tmp_path / "shared" / "timeline.log").read_text().splitlines()
    got = [json.loads(l)["i"] for l in lines]
    assert got == list(range(60)), "the mirror keeps the full history across local rotation"
    assert json.loads((tmp_path / "shared" / "meta.json").read_text())["pid"] == os.getpid()
    assert os.path.getsize(os.path.join(d, "timeline.log")) < 1500  # local copy stays bounded


def test_scalar_drain():
    from flodl_b200.monitor.telemetry import drain_scalars, record_scalar
    record_scalar("acc", 0.5)
    record_scalar("acc", 1.0)
    assert drain_scalars() == {"acc": 0.75} and drain_scalars() == {}


def test_timeline_html_and_verbose_build(tmp_path, capsys):
    from flodl_b200.monitor.monitor import Timeline
    tl = Timeline(0.01).start()
    tl.event("sync", round=1)
    time.sleep(0.05)
    tl.event("anchor", value=4)
    tl.stop()
    tl.save_html(str(tmp_path / "t.html"))
    text = (tmp_path / "t.html").read_text()
    assert "<svg" in text and "anchor" in text
    from flodl_b200.graph import FlowBuilder
    from flodl_b200.nn import Linear
    from flodl_b200.utils import log
    old = log.verbosity()
    log.set_verbosity(log.Verbosity.VERBOSE)
    try:
        FlowBuilder.from_(Linear(2, 2)).build()
    finally:
        log.set_verbosity(old)
    assert "Graph" in capsys.readouterr().err
