"""Per-host relay fold, single-port mux, status board and bind diagnosis
(reference: relay/agent_tests.rs, relay/mux_tests.rs, port_mux_tests.rs,
status.rs tests, bind_diag.rs tests)."""
import json
import os
import socket
import threading
import time
import urllib.request

import pytest
import torch

from flodl_b200.parallel.cpu_reduce import MAGIC, CpuReduceClient, CpuReduceController
from flodl_b200.parallel.membership import StartMode
from flodl_b200.parallel.portmux import PortMux, StatusBoard, describe_port_holder, port_holders
from flodl_b200.parallel.relay import RelayAgent
from flodl_b200.parallel.rendezvous import MAGIC_RDV, RendezvousServer, rendezvous

KEY = b"relay-test-key"


def _round(clients, vals, masses, rnd):
    out = [None] * len(clients)

    def run(i):
        out[i] = clients[i].all_reduce_scaled(vals[i], masses[i], rnd=rnd, timeout=20)

    ts = [threading.Thread(target=run, args=(i,)) for i in range(len(clients))]
    [t.start() for t in ts]
    [t.join() for t in ts]
    return out


def _wait(pred, t=10.0):
    end = time.time() + t
    while time.time() < end and not pred():
        time.sleep(0.02)
    return pred()


def test_relay_folds_host_ranks_into_one_upstream_frame():
    ctl = CpuReduceController(4, KEY, heartbeat_timeout=30)
    ra = RelayAgent(("127.0.0.1", ctl.port), KEY)
    rb = RelayAgent(("127.0.0.1", ctl.port), KEY)
    clients = [CpuReduceClient(r, "127.0.0.1", (ra if r < 2 else rb).port, KEY, heartbeat_s=0.2)
               for r in range(4)]
    assert _wait(lambda: len(ctl.conns) == 4)
    vals = [torch.full((4096,), float(r + 1)) for r in range(4)]
    masses = [1.0, 3.0, 2.0, 2.0]
    expect = sum((r + 1) * m for r, m in enumerate(masses)) / sum(masses)
    for rnd in (1, 2):
        for o in _round(clients, vals, masses, rnd):
            torch.testing.assert_close(o, torch.full((4096,), expect))
    # one data frame per host per round reached the controller
    assert ctl.frames_in == 4 and ra.frames_up == 2 and rb.frames_up == 2
    # heartbeats of relayed ranks are forwarded with their rank
    assert _wait(lambda: all(time.time() - ctl.last_hb[r] < 5 for r in range(4)))
    [c.close() for c in clients]
    ra.close(), rb.close(), ctl.close()


def test_relay_local_rank_exit_is_reported_and_round_completes():
    ctl = CpuReduceController(3, KEY, heartbeat_timeout=60)
    ra = RelayAgent(("127.0.0.1", ctl.port), KEY)
    clients = [CpuReduceClient(r, "127.0.0.1", ra.port if r < 2 else ctl.port, KEY,
                               heartbeat_s=0.2) for r in range(3)]
    assert _wait(lambda: len(ctl.conns) == 3)
    clients[1].close()  # a local rank leaves: the relay reports it upstream
    assert _wait(lambda: 1 in ctl.dead), "controller did not learn of the exit"
    vals = [torch.full((64,), 2.0), torch.full((64,), 6.0)]
    out = _round([clients[0], clients[2]], vals, [1.0, 1.0], rnd=7)
    for o in out:
        torch.testing.assert_close(o, torch.full((64,), 4.0))
    assert _wait(lambda: 1 in clients[0].dead), "DEAD was not fanned out by the relay"
    clients[0].close(), clients[2].close()
    ra.close(), ctl.close()


def test_port_mux_routes_rendezvous_reduce_and_http_on_one_port():
    mux = PortMux()
    rdv = RendezvousServer(2, KEY, port=None).start()
    ctl = CpuReduceController(2, KEY, port=None)
    board = StatusBoard()
    mux.route_magic(MAGIC_RDV, rdv.adopt)
    mux.route_magic(MAGIC, ctl.adopt)
    mux.serve_status(board)

    # rendezvous through the mux port
    res = [None, None]

    def join(i):
        res[i] = rendezvous("127.0.0.1", mux.port, KEY, rank=i, uid_fn=lambda: b"uid-xyz", timeout=20)

    ts = [threading.Thread(target=join, args=(i,)) for i in range(2)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    assert sorted(r.rank for r in res) == [0, 1] and all(r.uid == b"uid-xyz" for r in res)

    # CPU reduce through the same port
    clients = [CpuReduceClient(r, "127.0.0.1", mux.port, KEY, heartbeat_s=0.2) for r in range(2)]
    out = _round(clients, [torch.ones(8), torch.full((8,), 3.0)], [1.0, 1.0], rnd=1)
    torch.testing.assert_close(out[0], torch.full((8,), 2.0))

    # status over HTTP on the same port
    url = f"http://127.0.0.1:{mux.port}"
    with pytest.raises(urllib.error.HTTPError) as e:
        urllib.request.urlopen(url + "/state.json", timeout=5)
    assert e.value.code == 503
    board.publish({"phase": "running", "world": 2, "hosts": ["a"]})
    st = json.loads(urllib.request.urlopen(url + "/state.json", timeout=5).read())
    assert st["phase"] == "running" and st["world"] == 2 and not st["start_requested"]

    # operator start switch: refused under Auto, armed from loopback under Manual
    req = urllib.request.Request(url + "/start", method="POST", data=b"")
    with pytest.raises(urllib.error.HTTPError) as e:
        urllib.request.urlopen(req, timeout=5)
    assert e.value.code == 409
    board.configure_start(StartMode.Manual, "ab" * 16)
    assert urllib.request.urlopen(req, timeout=5).status == 200
    assert board.start_requested()

    # a remote peer without the token is refused; with it, accepted
    board2 = StatusBoard()
    board2.configure_start(StartMode.Hybrid, "cd" * 16)
    assert board2.request_start("10.0.0.5", "")[0] == 403
    assert board2.request_start("10.0.0.5", "cd" * 16)[0] == 200

    # unknown channel magic: dropped, the mux keeps serving
    s = socket.create_connection(("127.0.0.1", mux.port))
    s.sendall(b"XXXXjunk")
    assert _wait(lambda: mux.dropped >= 1)
    s.close()
    assert urllib.request.urlopen(url + "/healthz", timeout=5).read() == b"ok"
    [c.close() for c in clients]
    ctl.close(), mux.close()


def test_bind_diagnosis_names_the_holder():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    s.listen(1)
    port = s.getsockname()[1]
    assert any(pid == os.getpid() for pid, _ in port_holders(port))
    assert f"pid {os.getpid()}" in describe_port_holder(port)
    s.close()


def test_bind_diagnosis_message_from_port_mux():
    s = socket.socket()
    s.bind(("0.0.0.0", 0))
    s.listen(1)
    port = s.getsockname()[1]
    # SO_REUSEADDR does not allow two listeners on one port
    with pytest.raises(OSError, match="busy"):
        PortMux("127.0.0.1", port)
    s.close()


def test_broadcast_through_a_relay():
    ctl = CpuReduceController(3, KEY)
    ra = RelayAgent(("127.0.0.1", ctl.port), KEY)
    clients = [CpuReduceClient(r, "127.0.0.1", ra.port if r < 2 else ctl.port, KEY, heartbeat_s=0.2)
               for r in range(3)]
    assert _wait(lambda: len(ctl.conns) == 3)
    src = torch.randn(33)
    out = [None] * 3

    def run(r):
        out[r] = clients[r].broadcast_from_root(src.clone() if r == 2 else torch.zeros(33), root=2,
                                                rnd=0, timeout=20)

    ts = [threading.Thread(target=run, args=(r,)) for r in range(3)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    for o in out:
        torch.testing.assert_close(o, src)
    [c.close() for c in clients]
    ra.close(), ctl.close()
