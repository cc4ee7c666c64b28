"""Rendezvous, membership ledger and the local launcher (CPU ranks, gloo)."""
import json
import os
import sys
import threading

import pytest

from flodl_b200.parallel.launcher import LocalLauncher, Role, role_from_env
from flodl_b200.parallel.membership import ClusterPhase, JoinWindow, StartMode
from flodl_b200.parallel.rendezvous import RendezvousServer, rendezvous

HERE = os.path.dirname(os.path.abspath(__file__))


def test_rendezvous_assigns_ranks_and_relays_uid():
    key = b"k" * 32
    srv = RendezvousServer(3, key).start()
    out = {}

    def join(i, want):
        out[i] = rendezvous(srv.host, srv.port, key, rank=want, uid_fn=lambda: b"UID-123")

    ts = [threading.Thread(target=join, args=(i, w)) for i, w in enumerate([-1, 2, -1])]
    for t in ts:
        t.start()
    for t in ts:
        t.join(30)
    assert srv.wait(10) and srv.error is None
    ranks = sorted(r.rank for r in out.values())
    assert ranks == [0, 1, 2] and out[1].rank == 2
    assert all(r.uid == b"UID-123" and r.world == 3 for r in out.values())


def test_rendezvous_rejects_wrong_key_and_times_out():
    srv = RendezvousServer(2, b"a" * 32, idle_timeout=1.0).start()
    with pytest.raises(Exception):
        rendezvous(srv.host, srv.port, b"b" * 32, timeout=5)
    assert srv.wait(10)
    assert srv.rejected >= 1 and "idle" in (srv.error or "")


def test_join_window_modes_and_shrink():
    w = JoinWindow(2, StartMode.Auto)  # two members (hosts); b brings two devices
    assert w.join("a") and w.join("b", devices=2)
    assert not w.join("a")  # duplicate
    assert w.phase is ClusterPhase.Running and w.world == 3
    assert not w.join("c")  # formed
    w.remove("b", "heartbeat stale")
    assert w.world == 1 and w.phase is ClusterPhase.Shrinking
    assert w.partition(10) == {"a": range(0, 10)}
    m = JoinWindow(4, StartMode.Manual, min_size=2)
    m.join("x")
    assert not m.start()
    m.join("y")
    assert m.start() and m.world == 2
    h = JoinWindow(4, StartMode.Hybrid, min_size=1, window_s=0.0)
    h.join("p")
    assert h.poll() is ClusterPhase.Running


def test_role_from_env():
    assert role_from_env({}) is Role.SingleDevice
    assert role_from_env({"WORLD_SIZE": "4"}) is Role.Rank
    assert role_from_env({"FLODL_INTERNAL_ROLE": "relay"}) is Role.Relay


def test_launcher_runs_ranks(tmp_path):
    r = LocalLauncher([sys.executable, os.path.join(HERE, "rank_prog.py")], ["cpu"] * 3,
                      env={"OUT_DIR": str(tmp_path)}, timeout_s=120).run()
    assert r.ok and r.world == 3
    res = [json.load(open(tmp_path / f"rank{i}_attempt0.json")) for i in range(3)]
    assert all(x["sum"] == 6.0 for x in res)


def test_launcher_elastic_shrink_after_rank_failure(tmp_path):
    log = tmp_path / "deaths.jsonl"
    r = LocalLauncher([sys.executable, os.path.join(HERE, "rank_prog.py")], ["cpu"] * 3,
                      policy="shrink", env={"OUT_DIR": str(tmp_path), "FAIL_RANK": "1",
                                            "FAIL_ATTEMPT": "0"},
                      timeout_s=120, death_log=str(log)).run()
    assert r.ok and r.world == 2 and r.attempts == 2
    assert r.deaths[0]["exit_code"] == 3 and r.deaths[0]["local_rank"] == 1
    res = [json.load(open(tmp_path / f"rank{i}_attempt1.json")) for i in range(2)]
    assert all(x["sum"] == 3.0 and x["world"] == 2 for x in res)
    assert json.loads(log.read_text().splitlines()[0])["reason"] == "rank exited with an error"
