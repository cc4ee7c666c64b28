"""Communicator layer over gloo ranks, CPU worker, Rng (reference:
nccl_tests.rs host-side parts, worker.rs, rng.rs)."""
import json
import os
import subprocess
import sys

import pytest

from flodl_b200.parallel.nccl import NcclUniqueId
from flodl_b200.utils.worker import CpuWorker, Rng

HERE = os.path.dirname(__file__)


def test_rank_comm_collectives_split_and_abort_on_gloo():
    uid = NcclUniqueId.new()
    world = 4
    env = dict(os.environ, PYTHONPATH=os.path.dirname(HERE))
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "nccl_rank_prog.py"), str(r), str(world),
                               uid.raw.hex()], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                              env=env) for r in range(world)]
    outs = []
    for p in procs:
        o, e = p.communicate(timeout=180)
        assert p.returncode == 0, e
        outs.append(json.loads(o.strip().splitlines()[-1]))
    for r, o in enumerate(outs):
        assert o["sum"] == [10.0] * 4
        assert o["premul"] == [sum(0.5 * (k + 1) * (k + 1) for k in range(world))] * 4
        assert o["bcast"] == [3.0, 3.0]
        assert o["per_rank"] == [0.0, 10.0, 20.0, 30.0]
        assert o["split"] == [r // 2, 2, 2.0 if r % 2 == 0 else 4.0]


def test_unique_id_is_128_bytes():
    u = NcclUniqueId.new()
    assert len(u.raw) == 128 and u.address()[0] == "127.0.0.1"
    with pytest.raises(ValueError):
        NcclUniqueId(b"short")


def test_cpu_worker_runs_in_order_and_reports_errors():
    w = CpuWorker()
    seen = []
    for i in range(50):
        w.submit(lambda i=i: seen.append(i))
    w.join()
    assert seen == list(range(50)) and w.done == 50
    w.submit(lambda: 1 / 0)
    with pytest.raises(ZeroDivisionError):
        w.join()
    w.close()


def test_rng_deterministic_unbiased_shuffle():
    a, b = Rng(7), Rng(7)
    assert [a.next_u64() for _ in range(5)] == [b.next_u64() for _ in range(5)]
    assert Rng(0).next_u64() == 0xE220A8397B1DCDAF  # SplitMix64 reference output for seed 0
    r = Rng(1)
    counts = [0] * 3
    for _ in range(30000):
        counts[r.below(3)] += 1
    assert all(abs(c - 10000) < 500 for c in counts)
    xs = Rng(3).shuffle(list(range(20)))
    assert sorted(xs) == list(range(20)) and xs != list(range(20))
    assert 0.0 <= Rng(5).uniform() < 1.0


def test_collective_trace_enter_exit(capsys):
    from flodl_b200.utils import log
    old = log.verbosity()
    log.set_verbosity(log.Verbosity.TRACE)
    try:
        with log.collective("all_reduce", numel=8):
            pass
        with pytest.raises(ValueError):
            with log.collective("broadcast"):
                raise ValueError("x")
    finally:
        log.set_verbosity(old)
    err = capsys.readouterr().err
    assert "ENTER all_reduce #" in err and "numel=8" in err and "EXIT all_reduce" in err
    assert "FAIL(ValueError) broadcast" in err
    with log.collective("quiet"):
        pass
    assert "quiet" not in capsys.readouterr().err
