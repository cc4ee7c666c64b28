"""LR-aware meta-controller (reference: lr_event_meta.rs tests)."""
import pytest

from flodl_b200.parallel.meta import LrEventMeta


def test_probe_never_acts_and_cosine_decay_is_quiet():
    m = LrEventMeta()
    assert m.observe(1.0, 10, "shrink", "probe") is None
    lr = 1.0
    for _ in range(20):
        lr *= 0.98
        assert m.observe(lr, 10, "ok", "stable") is None


def test_lr_cliff_threshold_boundary():
    m = LrEventMeta()
    m.observe(1.0, 100, "ok", "stable")
    assert m.observe(0.75, 100, "ok", "stable") is None      # 25% drop: under 30%
    m2 = LrEventMeta()
    m2.observe(1.0, 100, "ok", "stable")
    assert m2.observe(0.65, 100, "ok", "stable") == pytest.approx(0.5)  # 35%: fires at the base


def test_sustained_guard_pattern_by_phase():
    m = LrEventMeta()
    out = [m.observe(1.0, 50, "shrink", "mature") for _ in range(2)]
    assert out[0] is None and out[1] == pytest.approx(0.7)   # mature: K=2, base 0.7
    m = LrEventMeta()
    out = [m.observe(1.0, 50, "shrink", "warmup") for _ in range(5)]
    assert out[:4] == [None] * 4 and out[4] == pytest.approx(0.3)


def test_trend_softens_and_compound_clamps():
    m = LrEventMeta()
    for a in (100, 100, 100, 100):
        m.observe(1.0, a, "ok", "stable")
    f = m.observe(0.1, 50, "ok", "stable")    # anchor already shrinking: trend < 0 -> larger factor
    assert f > 0.5 and m.anchor_trend() < 0
    m = LrEventMeta()
    for _ in range(2):
        m.observe(1.0, 10, "shrink", "mature")
    f = m.observe(0.1, 10, "shrink", "mature")  # both watchers: 0.5 x 0.7
    assert f == pytest.approx(0.35)
    assert m.is_settled()
