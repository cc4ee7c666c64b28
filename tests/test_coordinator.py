"""Progressive dispatch, window ledger, callback roles, alerts (reference:
chunk_pool.rs tests, cluster_coordinator/tests)."""
import random

import pytest

from flodl_b200.monitor.records import RecordStore
from flodl_b200.parallel.coordinator import (AlertLane, CallbackRoles, ChunkPool, WindowLedger,
                                             spans_from_throughput)


def _covered(chunks):
    s = set()
    for off, n in chunks:
        rng = set(range(off, off + n))
        assert not (s & rng), "overlapping chunks"
        s |= rng
    return s


def test_spans_follow_throughput_and_cover_exactly():
    assert spans_from_throughput(100, [1, 3]) == [25, 75]
    assert sum(spans_from_throughput(101, [1, 1, 1])) == 101
    assert spans_from_throughput(10, [0, 0]) == [5, 5]


def test_owner_front_thief_tail_never_overlap_and_epoch_completes():
    p = ChunkPool(0, 1000, spans_from_throughput(1000, [1, 1, 2]))
    assert p.reservation(2) == (500, 500)
    rng = random.Random(0)
    taken = []
    speeds = [1, 3, 2]
    while True:
        r = rng.choices(range(3), weights=speeds)[0]
        c = p.take_chunk(37, r)
        if c is None:
            break
        taken.append(c)
        p.mark_completed(r, c[1])
    assert _covered(taken) == set(range(1000))
    assert p.is_epoch_done() and p.completed == 1000 and p.uncovered_ranges() == []


def test_forfeit_redispatches_dead_ranks_chunks_first():
    p = ChunkPool.equal(0, 100, 2)
    a = p.take_chunk(10, 1)
    assert a == (50, 10) and p.in_flight(1) == 10
    assert p.forfeit(1) == 50  # 10 in flight + 40 unassigned
    assert p.in_flight(1) == 0
    assert p.take_chunk(100, 0) == (50, 10)  # the hole closes first
    got = [(50, 10)]
    while (c := p.take_chunk(100, 0)) is not None:
        got.append(c)
    assert _covered(got) == set(range(100))


def test_rollback_rewinds_cursor_or_reclaims():
    p = ChunkPool.equal(0, 100, 2)
    c = p.take_chunk(20, 0)
    p.rollback_take(0, *c)
    assert p.reservation(0) == (0, 50) and p.in_flight(0) == 0
    c1 = p.take_chunk(20, 0)
    p.take_chunk(5, 1)
    with pytest.raises(ValueError):
        p.rollback_take(0, 99, 1)
    p.rollback_take(0, *c1)
    assert p.remaining() == 95


def test_coverage_snapshot_and_resume_hands_out_exactly_the_holes():
    p = ChunkPool.equal(3, 60, 3)
    c0 = p.take_chunk(10, 0)
    p.mark_completed(0, 10)
    p.take_chunk(10, 1)  # in flight: uncovered by design
    unc = p.uncovered_ranges()
    assert (c0[0], c0[1]) not in unc and sum(n for _, n in unc) == 50
    q = ChunkPool.from_coverage(3, 60, 3, unc)
    got = []
    while (c := q.take_chunk(7, 2)) is not None:
        got.append(c)
        q.mark_completed(2, c[1])
    assert _covered(got) == set(range(60)) - set(range(c0[0], c0[0] + 10)) and q.is_epoch_done()


def test_window_ledger_marginal_rate_excludes_fill_and_callbacks():
    L = WindowLedger(2)
    L.record_batch(0, 32, 50.0)  # first batch carries the fill
    for _ in range(4):
        L.record_batch(0, 32, 10.0)
    L.exclude(0, 0.0)
    assert L.per_batch_ms(0) == pytest.approx(10.0)
    assert L.fill_excess_ms(0) == pytest.approx(40.0)
    assert L.delivered_rate(0) == pytest.approx(3.2)
    assert L.per_batch_ms(1) is None
    L.reset()
    assert L.batches(0) == 0


def test_callback_roles_sticky_with_failover():
    roles = CallbackRoles(3, margin=0.1)
    assert roles.observe({0: 10.0, 1: 9.5, 2: 12.0}) == 0   # within the margin: sticky
    assert roles.observe({0: 10.0, 1: 8.0, 2: 12.0}) == 1   # clearly faster: moves
    assert roles.rank_died(1) == 0
    assert roles.observe({0: 10.0, 2: 5.0}) == 2


def test_alert_lane_collapses_and_publishes():
    store = RecordStore()
    lane = AlertLane(store, collapse_s=60, live_cap=2, log=lambda m: None)
    assert lane.raise_("rank_lost", "root/h/rank3", "heartbeat stale", now=0.0)
    assert lane.raise_("rank_lost", "root/h/rank3", "again", now=10.0) is None
    assert lane.live[("rank_lost", "root/h/rank3")]["repeats"] == 1
    lane.raise_("drift", "root", "anchor cut", now=11.0)
    lane.raise_("control_drop", "root", "missed rank 2", now=12.0)
    assert len(lane.live) == 2
    assert any(r.get("class") == "rank_lost" for r in store.history("root", 10))
    with pytest.raises(ValueError):
        lane.raise_("info", "root", "x")


def test_max_failure_threshold():
    from flodl_b200.parallel.coordinator import MaxFailureThreshold
    assert MaxFailureThreshold(absolute=3).limit_for(100) == 3
    assert MaxFailureThreshold(percent=0.2).limit_for(10) == 2
    assert MaxFailureThreshold(percent=0.2).limit_for(5) == 1
    assert MaxFailureThreshold(percent=1.5).limit_for(4) == 4
    assert MaxFailureThreshold(percent=0.0).breached(0, 8)
    assert not MaxFailureThreshold(absolute=2).breached(1, 4)
