"""Dial-in membership: agents join, receive envelopes, run and report ranks;
a failed rank aborts every host (reference: launcher/agent.rs,
membership_tests.rs)."""
import json
import os
import sys
import threading

from flodl_b200.parallel.agent import JoinServer, run_agent
from flodl_b200.parallel.membership import StartMode

HERE = os.path.dirname(__file__)
KEY = b"join-test-key-00"
ENV = {"PYTHONPATH": os.path.dirname(HERE)}  # shipped to the rank children in ASSIGN


def _agents(srv, out, hosts):
    rcs = {}

    def go(h, n):
        rcs[h] = run_agent(f"127.0.0.1:{srv.port}", KEY, devices=n, host=h, timeout_s=120,
                           log=lambda m: None)

    ts = [threading.Thread(target=go, args=hn) for hn in hosts]
    [t.start() for t in ts]
    [t.join(180) for t in ts]
    return rcs


def test_agents_join_form_and_run_ranks(tmp_path):
    cmd = [sys.executable, os.path.join(HERE, "agent_child.py"), str(tmp_path)]
    srv = JoinServer(KEY, 2, cmd, StartMode.Auto, env=ENV)
    rcs = _agents(srv, tmp_path, [("hostA", 2), ("hostB", 1)])
    assert rcs == {"hostA": 0, "hostB": 0}
    assert srv.wait(30)
    recs = sorted((json.loads(p.read_text()) for p in tmp_path.glob("rank*.json")), key=lambda r: r["rank"])
    assert [r["rank"] for r in recs] == [0, 1, 2] and all(r["world"] == 3 for r in recs)
    by_host = {r["rank"]: r["host"] for r in recs}
    assert len({by_host[0], by_host[1]}) == 1 or len({by_host[1], by_host[2]}) == 1
    assert sorted(e["rank"] for e in srv.exits) == [0, 1, 2]
    srv.close()


def test_failed_rank_aborts_all_hosts(tmp_path):
    cmd = [sys.executable, "-c", "import os,sys,time; r=int(os.environ['RANK']); "
           "sys.exit(5) if r == 0 else time.sleep(60)"]
    srv = JoinServer(KEY, 2, cmd, StartMode.Auto, policy="abort")
    rcs = _agents(srv, tmp_path, [("h1", 1), ("h2", 1)])
    assert not srv.wait(30) and "failed" in srv.aborted
    assert sorted(rcs.values()) in ([3, 5], [5, 3], [3, 3])
    srv.close()


def test_late_joiner_refused_after_formation(tmp_path):
    cmd = [sys.executable, "-c", "pass"]
    srv = JoinServer(KEY, 1, cmd, StartMode.Auto)
    rcs = _agents(srv, tmp_path, [("only", 1)])
    assert rcs["only"] == 0
    rc = run_agent(f"127.0.0.1:{srv.port}", KEY, devices=1, host="late", log=lambda m: None)
    assert rc == 2 and any("formed" in r[1] for r in srv.window.refused)
    srv.close()
