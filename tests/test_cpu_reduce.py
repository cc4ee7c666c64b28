"""CPU averaging controller/client over signed frames, heartbeats and dead-rank
detection with fake ranks (reference: cpu_reduce_tests.rs, controller_tests.rs,
cluster_coordinator/tests/heartbeat.rs)."""
import threading
import time

import pytest
import torch

from flodl_b200._ext import native
from flodl_b200.parallel.cpu_reduce import CpuReduceClient, CpuReduceController

KEY = b"test-session-key"


def test_frames_sign_and_reject_tampering():
    N = native()
    f = N.encode_frame(0x12345678, 2, 9, b"payload", KEY)
    assert N.decode_frame(f, KEY)[4] == b"payload"
    bad = bytearray(f)
    bad[30] ^= 1
    with pytest.raises(RuntimeError, match="signature"):
        N.decode_frame(bytes(bad), KEY)
    with pytest.raises(RuntimeError, match="signature"):
        N.decode_frame(f, b"other-key")
    with pytest.raises(RuntimeError, match="ceiling"):
        N.decode_frame(f, KEY, 3)


def test_weighted_round_three_ranks():
    ctl = CpuReduceController(3, KEY)
    clients = [CpuReduceClient(r, "127.0.0.1", ctl.port, KEY, heartbeat_s=0.2) for r in range(3)]
    vals = [torch.full((1000,), float(r)) for r in range(3)]
    masses = [1.0, 2.0, 5.0]
    out = [None] * 3

    def run(r):
        out[r] = clients[r].all_reduce_scaled(vals[r], masses[r], rnd=1, timeout=20)

    ts = [threading.Thread(target=run, args=(r,)) for r in range(3)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    expect = sum(r * m for r, m in zip(range(3), masses)) / sum(masses)
    for o in out:
        torch.testing.assert_close(o, torch.full((1000,), expect))
    [c.close() for c in clients]
    ctl.close()


def test_bf16_wire_roundtrip():
    ctl = CpuReduceController(1, KEY)
    c = CpuReduceClient(0, "127.0.0.1", ctl.port, KEY, bf16_wire=True)
    x = torch.randn(513)
    y = c.all_reduce_scaled(x, 1.0, rnd=5, timeout=10)
    torch.testing.assert_close(y, x.bfloat16().float())
    c.close()
    ctl.close()


def test_dead_rank_is_dropped_and_round_completes():
    ctl = CpuReduceController(2, KEY, heartbeat_timeout=0.6)
    a = CpuReduceClient(0, "127.0.0.1", ctl.port, KEY, heartbeat_s=0.1)
    b = CpuReduceClient(1, "127.0.0.1", ctl.port, KEY, heartbeat_s=0.1)
    time.sleep(0.3)
    b.stop_heartbeat()  # rank 1 hangs: no heartbeat, never contributes
    out = a.all_reduce_scaled(torch.ones(10) * 3, 1.0, rnd=2, timeout=10)
    torch.testing.assert_close(out, torch.full((10,), 3.0))
    assert 1 in ctl.dead and 1 in a.dead
    a.close()
    b.close()
    ctl.close()


def test_reduce_scaled_native_matches_python():
    ts = [torch.randn(100000) for _ in range(4)]
    ms = [1.0, 2.0, 3.0, 4.0]
    out = native().reduce_scaled(ts, ms)
    torch.testing.assert_close(out, sum(ts) / sum(ms))


def test_broadcast_from_root():
    ctl = CpuReduceController(3, KEY)
    clients = [CpuReduceClient(r, "127.0.0.1", ctl.port, KEY, heartbeat_s=0.2) for r in range(3)]
    src = torch.randn(257)
    out = [None] * 3

    def run(r):
        t = src.clone() if r == 1 else torch.zeros(257)
        out[r] = clients[r].broadcast_from_root(t, root=1, rnd=-5, timeout=20)

    ts = [threading.Thread(target=run, args=(r,)) for r in range(3)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    for o in out:
        torch.testing.assert_close(o, src)
    [c.close() for c in clients]
    ctl.close()
