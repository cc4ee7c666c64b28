"""Coordinator-driven runtime on CPU ranks (gloo), fault handling on the host,
and the native ElChe's protocol (reference: cluster_worker_tests.rs
end-to-end smokes, cluster_coordinator/tests/heartbeat.rs, ddp_tests.rs
ElChe tests). Failures are made on the host only: a rank that leaves between
windows, a rank that stops heart-beating, a slowed rank."""
import multiprocessing as std_mp
import os
import socket

import pytest
import torch

from flodl_b200.data import TensorDataSet
from flodl_b200.nn import Linear
from flodl_b200.optim import SGD
from flodl_b200.parallel import ElCheConfig, ElCheMode, Trainer, TrainerConfig


def make_model(device):
    torch.manual_seed(0)
    return Linear(4, 1, device=device)


def make_opt(params):
    return SGD(params, 0.05)


def train_fn(model, batch):
    x, y = batch
    return torch.nn.functional.mse_loss(model(x), y)


def _dataset(n=512):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(n, 4, generator=g)
    w = torch.tensor([[1.0], [-2.0], [0.5], [3.0]])
    return TensorDataSet(x, x @ w)


def _builder(mode, world, epochs, anchor=2, hb=30.0, **ec):
    e = ElCheConfig().mode(mode).anchor(anchor)
    for k, v in ec.items():
        setattr(e, k + "_", v)
    cfg = TrainerConfig().batch_size(16).num_epochs(epochs).elche(e).heartbeat_timeout_secs(hb)
    return (Trainer.builder(make_model, make_opt, train_fn).dataset(_dataset()).config(cfg)
            .devices(["cpu"] * world))


def test_cadence_via_coordinator_balances_a_slow_rank():
    st = (_builder(ElCheMode.NcclCadence, 2, 3, anchor=2, divergence_guard_=False)
          .test_hooks(slow_ms_per_batch={1: 25.0}).run().join(timeout=300))
    rec = st.record
    assert st.syncs > 0 and rec["syncs"] == st.syncs
    late = rec["batch_counts"][-1]
    assert late[0] > late[1], f"the slow rank should get fewer batches: {rec['batch_counts']}"
    assert st.losses[-1] < st.losses[0]


def test_sync_via_coordinator_one_batch_windows():
    st = _builder(ElCheMode.NcclSync, 2, 2).run().join(timeout=300)
    assert all(c == [1, 1] for c in st.record["batch_counts"])
    assert st.losses[-1] < st.losses[0]


def test_cpu_backend_via_coordinator_hosted_reducer():
    st = _builder(ElCheMode.CpuCadence, 2, 2).run().join(timeout=300)
    assert st.syncs > 0 and st.losses[-1] < st.losses[0]


def test_cpu_async_overshoots_a_bounded_number_of_batches():
    st = (_builder(ElCheMode.CpuAsync, 2, 2, anchor=2, max_overshoot=2, divergence_guard_=False)
          .test_hooks(slow_ms_per_batch={1: 30.0}).run().join(timeout=300))
    assert st.record["overshoot"] > 0
    assert st.record["overshoot"] <= 2 * st.record["syncs"]


def test_rank_leaving_between_windows_survivors_reform_and_finish():
    st = (_builder(ElCheMode.NcclCadence, 3, 3).test_hooks(leave_after_syncs={2: 2})
          .group_timeout(20).run().join(timeout=300))
    rec = st.record
    assert [d["rank"] for d in rec["deaths"]] == [2]
    assert rec["deaths"][0]["why"] == "left"
    assert rec["sessions"] >= 2  # the first session and the survivors' re-formation
    assert rec["epochs"][-1]["alive"] == [0, 1]
    assert st.losses[-1] < st.losses[0]


def test_rank_that_stops_heartbeating_is_declared_dead_and_round_retried():
    st = (_builder(ElCheMode.NcclCadence, 3, 2, hb=1.5).test_hooks(hang_after_windows={1: 2})
          .group_timeout(4).run().join(timeout=300))
    rec = st.record
    assert [d["rank"] for d in rec["deaths"]] == [1]
    assert rec["deaths"][0]["why"] == "heartbeat stale"
    assert rec["retries"] >= 1
    assert rec["epochs"][-1]["alive"] == [0, 2]


# ------------------------------------------------------------------ averager semantics
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _BNNet(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.lin = torch.nn.Linear(3, 3)
        self.bn = torch.nn.BatchNorm1d(3)


def _averager_worker(rank, world, port, batches, alpha, q):
    import torch.distributed as dist

    from flodl_b200.parallel.config import AverageBackend
    from flodl_b200.parallel.trainer import _Averager

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    net = _BNNet()
    with torch.no_grad():
        for p in net.parameters():
            p.fill_(float(rank + 1))
        net.bn.running_mean.fill_(10.0 * (rank + 1))
        net.bn.running_var.fill_(float(rank + 1))
    avg = _Averager(net, None, AverageBackend.NCCL, rank, world, torch.device("cpu"),
                    gamma=1.0, easgd_alpha=alpha)
    avg.average(batches[rank])
    # plain lists: a tensor in the queue is shared through a file descriptor
    # that dies with this process, which may exit before the parent reads it
    q.put((rank, [p.detach().tolist() for p in net.parameters()],
           net.bn.running_mean.tolist(), net.bn.running_var.tolist()))
    dist.destroy_process_group()


def _run_averager(batches, alpha=None):
    world = len(batches)
    ctx = std_mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_averager_worker, args=(r, world, port, batches, alpha, q))
          for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for r, params, rm, rv in [q.get(timeout=120) for _ in range(world)]:
        out[r] = ([torch.tensor(p) for p in params], torch.tensor(rm), torch.tensor(rv))
    for p in ps:
        p.join(timeout=60)
    return out


def test_buffers_averaged_over_movers_params_by_work():
    # rank 0 did 1 batch, rank 1 did 3, rank 2 was idle
    out = _run_averager([1, 3, 0])
    want_param = (1 * 1.0 + 3 * 2.0) / 4.0
    for r in range(3):
        params, rm, rv = out[r]
        for p in params:
            assert torch.allclose(p, torch.full_like(p, want_param))
        # buffers: equal weight over the ranks that moved (0 and 1), the idle one excluded
        assert torch.allclose(rm, torch.full_like(rm, (10.0 + 20.0) / 2))
        assert torch.allclose(rv, torch.full_like(rv, (1.0 + 2.0) / 2))


def test_easgd_blend_is_one_minus_alpha_local_plus_alpha_center():
    out = _run_averager([2, 2], alpha=0.25)
    center = 1.5
    for r in range(2):
        params, _, _ = out[r]
        local = float(r + 1)
        for p in params:
            assert torch.allclose(p, torch.full_like(p, 0.75 * local + 0.25 * center))


def test_all_idle_round_changes_nothing():
    out = _run_averager([0, 0])
    for r in range(2):
        params, rm, _ = out[r]
        for p in params:
            assert torch.allclose(p, torch.full_like(p, float(r + 1)))
        assert torch.allclose(rm, torch.full_like(rm, 10.0 * (r + 1)))


# ------------------------------------------------------------------ native ElChe protocol
def _elche(world=2, anchor=10):
    from flodl_b200._ext import native
    return native().ElChe(world, anchor)


def test_elche_growth_is_proposed_then_committed_vetoed_or_discarded():
    e = _elche(2, 4)
    e.set_overhead_target(0.05)
    for _ in range(6):  # reach Stable with an expensive reduce
        e.report_timing([40.0, 40.0], [4, 4], 20.0)
        e.apply_verdict("stable", 1.0, False)
    a = e.anchor()
    e.report_timing([10.0 * a, 10.0 * a], [a, a], 200.0)
    p = e.proposed_anchor()
    assert p > a, "an overhead above target must propose growth"
    assert e.anchor() == a, "a proposal is not applied before a verdict"
    e.commit_proposed_anchor()
    assert e.anchor() == p
    e.report_timing([10.0 * p, 10.0 * p], [p, p], 200.0)
    assert e.proposed_anchor() > p
    e.veto_proposed_growth()
    assert e.anchor() == p and not e.growth_enabled()
    e.report_timing([10.0 * p, 10.0 * p], [p, p], 200.0)
    assert e.proposed_anchor() == 0, "growth stays latched off after a veto"
    for _ in range(5):
        e.commit_proposed_anchor()
    assert e.growth_enabled(), "five consecutive stable verdicts re-arm growth"
    e.apply_verdict("nudge", 0.5, False)
    assert e.anchor() == max(1, -(-p // 2))


def test_elche_dead_window_escape_drops_a_silent_pinned_anchor():
    e = _elche(3, 4)
    e.set_initial_anchor(2)
    for _ in range(4):
        e.report_timing([40.0, 80.0, 0.0], [4, 4, 0], 1.0)
    assert e.anchor_rank() == 2
    e.report_timing([40.0, 80.0, 0.0], [4, 4, 0], 1.0)
    assert e.anchor_rank() == 1, "after 5 empty reports the slowest reporting rank takes over"


def test_elche_state_round_trip_and_world_check():
    e = _elche(2, 5)
    for _ in range(7):
        e.report_timing([50.0, 25.0], [5, 5], 1.0)
    st = e.to_state()
    assert st["phase"] == "stable" and st["calibration_count"] == 7
    f = _elche(2, 1)
    f.restore_from_state(st)
    assert f.anchor() == e.anchor() and f.anchor_rank() == e.anchor_rank()
    assert f.phase() == "stable" and f.batch_counts() == e.batch_counts()
    g = _elche(3, 1)
    with pytest.raises(Exception):
        g.restore_from_state(st)


def test_elche_partition_ratios_fix_the_split():
    e = _elche(2, 4)
    e.set_partition_ratios([0.75, 0.25])
    assert e.batch_counts() == [12, 4] and e.anchor_rank() == 1
    for _ in range(6):  # measured speeds do not rebalance explicit ratios
        e.report_timing([10.0, 90.0], [12, 4], 1.0)
    assert e.batch_counts()[0] == 3 * e.batch_counts()[1]
    with pytest.raises(Exception):
        e.set_partition_ratios([0.5, 0.6])


def test_elche_relax_up_honours_max_batch_diff():
    e = _elche(2, 4)
    e.set_max_batch_diff(4)
    e.report_timing([40.0, 40.0], [4, 8], 0.0)  # rank 1 is twice as fast
    e.relax_anchor_up()  # anchor 5 -> fast 10: diff 5 > 4, refused
    assert e.anchor() == 4
    f = _elche(2, 3)
    f.set_max_batch_diff(4)
    f.report_timing([30.0, 30.0], [3, 6], 0.0)
    f.relax_anchor_up()  # anchor 4 -> fast 8: diff 4, allowed
    assert f.anchor() == 4


def test_elche_window_cap_scales_to_one_epoch():
    e = _elche(2, 10)
    e.set_max_total(12)
    e.report_timing([100.0, 25.0], [10, 10], 1.0)
    assert sum(e.batch_counts()) == 12 and e.window_cap_binding()


def test_rank_report_crosses_the_queue_by_value():
    """A rank's report travels to the parent as bytes (dtype, shape, data), so
    it survives the rank process exiting before the parent reads it."""
    import pickle

    from flodl_b200.parallel.trainer import TrainedState, _report_as_tensors, _report_by_value

    p = [("w", torch.randn(3, 4)), ("h", torch.randn(5).bfloat16())]
    st = TrainedState(params=list(p), buffers=[("n", torch.tensor(7))])
    back = _report_as_tensors(pickle.loads(pickle.dumps(_report_by_value(st))))
    for (n0, t0), (n1, t1) in zip(p, back.params):
        assert n0 == n1 and t0.dtype == t1.dtype and torch.equal(t0, t1)
    assert back.buffers[0][1].item() == 7
