"""FlowBuilder / Graph behaviour (reference: flodl/src/graph/tests, tree_tests.rs)."""
import pytest
import torch

from flodl_b200.graph import FlowBuilder, MergeOp, SoftmaxRouter, ThresholdHalt, FixedSelector
from flodl_b200.nn import GELU, Identity, LayerNorm, Linear, Module, NamedInputModule, ReLU


def test_sequential_and_residual():
    torch.manual_seed(0)
    l1, ln, l2, l3 = Linear(4, 8), LayerNorm(8), Linear(8, 8), Linear(8, 2)
    g = FlowBuilder.from_(l1).through(GELU()).through(ln).also(l2).through(l3).build()
    x = torch.randn(3, 4)
    h = ln(torch.nn.functional.gelu(l1(x)))
    ref = l3(h + l2(h))
    torch.testing.assert_close(g(x), ref)
    names = [n for n, _ in g.graph_named_parameters()]
    # node ids share one counter across node kinds, as the reference's builder
    # numbers them (linear_1, gelu_2, layernorm_3, linear_4, add_5, linear_6)
    assert names == ["linear_1/weight", "linear_1/bias", "layernorm_3/weight", "layernorm_3/bias",
                     "linear_4/weight", "linear_4/bias", "linear_6/weight", "linear_6/bias"]


def test_tag_names_parameters_and_tagged_values():
    g = FlowBuilder.from_(Linear(4, 4)).tag("enc").through(ReLU()).tag("act").through(Linear(4, 2)).build()
    names = [n for n, _ in g.graph_named_parameters()]
    assert names[0] == "enc/weight" and names[-1] == "linear_3/bias"
    x = torch.randn(2, 4)
    g(x)
    assert torch.all(g.tagged("act") >= 0)


def test_split_merge_mean_and_add():
    a, b = Linear(3, 3), Linear(3, 3)
    x = torch.randn(5, 3)
    g = FlowBuilder.new().split([a, b]).merge(MergeOp.MEAN).build()
    torch.testing.assert_close(g(x), (a(x) + b(x)) / 2)
    g2 = FlowBuilder.new().split([a, b]).merge(MergeOp.ADD).build()
    torch.testing.assert_close(g2(x), a(x) + b(x))


def test_builder_errors_surface_at_build():
    fb = FlowBuilder.new().split([Linear(2, 2), Linear(2, 2)]).through(Linear(2, 2))
    with pytest.raises(ValueError, match="single stream"):
        fb.build()
    with pytest.raises(ValueError, match="duplicate tag"):
        FlowBuilder.new().tag("a").through(Identity()).tag("a").build()
    with pytest.raises(ValueError, match="unresolved forward"):
        FlowBuilder.new().through(Linear(2, 2)).using(["later"]).build()


class _Cross(NamedInputModule):
    NAME = "cross"

    def forward_named(self, x, refs):
        return x * 0 + sum(refs.values())


def test_using_backward_and_forward_refs():
    g = (FlowBuilder.from_(Linear(2, 2)).tag("h").through(Linear(2, 2)).through(_Cross()).using(["h"])
         .build())
    x = torch.randn(3, 2)
    out = g(x)
    torch.testing.assert_close(out, g.tagged("h"))
    # forward reference: reads the previous call's value (None on the first call)
    g2 = FlowBuilder.new().through(_Cross()).using(["state"]).through(Linear(2, 2)).tag("state").build()
    assert g2.has_state() is False
    y1 = g2(torch.randn(1, 2))
    assert g2.has_state()
    y2 = g2(torch.randn(1, 2))
    assert y1.shape == y2.shape


def test_input_ports_multi_input():
    g = FlowBuilder.from_(Identity()).input(["aux"]).through(_Cross()).using(["aux"]).build()
    a, b = torch.randn(2, 3), torch.randn(2, 3)
    torch.testing.assert_close(g(a, b), b)


def test_loops_for_while_until():
    body = Linear(2, 2)
    g = FlowBuilder.new().loop_body(body).for_n(3).build()
    x = torch.randn(1, 2)
    torch.testing.assert_close(g(x), body(body(body(x))))
    ctr = {"n": 0}

    class Cond(Module):
        def forward(self, x):
            ctr["n"] += 1
            return torch.tensor(1.0 if ctr["n"] <= 2 else -1.0)

    g2 = FlowBuilder.new().loop_body(Identity()).while_cond(Cond(), 10).build()
    g2(x)
    assert ctr["n"] == 3
    g3 = FlowBuilder.new().loop_body(Identity()).until_cond(ThresholdHalt(-100.0), 5).build()
    g3(x)
    assert g3.traces_by_node("loop_2") is not None and len(g3.traces_by_node("loop_2")) == 1


def test_gate_and_switch():
    torch.manual_seed(1)
    e1, e2 = Linear(4, 4), Linear(4, 4)
    router = SoftmaxRouter(4, 2)
    g = FlowBuilder.new().gate(router, [e1, e2]).build()
    x = torch.randn(3, 4)
    w = router(x)
    ref = e1(x) * w[:, :1] + e2(x) * w[:, 1:]
    torch.testing.assert_close(g(x), ref)
    s = FlowBuilder.new().switch(FixedSelector(1), [e1, e2]).build()
    torch.testing.assert_close(s(x), e2(x))


def test_map_each_and_slices():
    body = Linear(3, 3)
    x = torch.randn(4, 3)
    g = FlowBuilder.new().map(body).each().build()
    torch.testing.assert_close(g(x), body(x))
    g2 = FlowBuilder.new().map(Identity()).slices(3).build()
    torch.testing.assert_close(g2(x), x)


def test_structural_hash_stable_and_sensitive():
    def mk(n):
        torch.manual_seed(0)
        return FlowBuilder.from_(Linear(4, n)).through(GELU()).through(Linear(n, 2)).build()
    h1, h2, h3 = mk(8).structural_hash(), mk(8).structural_hash(), mk(9).structural_hash()
    assert h1 == h2 and h1 != h3 and len(h1) == 64


def test_graph_tree_paths_freeze_thaw():
    inner = FlowBuilder.from_(Linear(4, 4)).tag("proj").through(GELU()).label("encoder").build()
    outer = FlowBuilder.from_(inner).through(Linear(4, 2)).tag("head").build()
    assert outer.child_graph("encoder") is inner
    assert outer.validate_path("encoder") == "graph"
    assert outer.validate_path("encoder.proj") == "tag"
    outer.freeze("encoder")
    assert outer.is_frozen("encoder") and not outer.is_frozen("head")
    outer.thaw("encoder")
    assert not outer.is_frozen("encoder")
    assert len(outer.parameters_at("encoder.proj")) == 2


def test_observe_collect_flush_trend():
    g = FlowBuilder.from_(Identity()).tag("x").build()
    for v in [5.0, 4.0, 3.0, 2.0]:
        g(torch.full((2,), v))
        g.collect(["x"])
        g.flush(["x"])
    t = g.trend("x")
    assert t.improving(0) and t.slope(0) == pytest.approx(-1.0)
    assert not t.stalled(0, 0.5)


def test_dot_export():
    g = FlowBuilder.from_(Linear(2, 2)).tag("a").also(Linear(2, 2)).build()
    d = g.dot()
    assert d.startswith("digraph") and '"linear_1" -> "linear_2"' in d


def test_quickstart_mlp_flowbuilder_learns():
    """BASELINE config 1 (CPU FlowBuilder MLP regression), shortened."""
    from flodl_b200.examples.mlp_flowbuilder import run
    r = run(steps=300)
    assert r["final_loss"] < 0.3 * r["first_loss"], r


def test_profiling_levels_stats_trends_and_viz(tmp_path):
    """Per-node timing, levels and parallelism, statistics, timing trends,
    heatmap, HTML plots, CSV/log export (reference: graph/profile.rs,
    heatmap.rs, plot.rs tests)."""
    a, b = Linear(16, 16), Linear(16, 16)
    g = (FlowBuilder.from_(Linear(8, 16)).tag("enc").split([a, b]).merge(MergeOp.ADD)
         .through(Linear(16, 4)).tag("head").build())
    g.enable_profiling()
    x = torch.randn(32, 8)
    for i in range(3):
        g(x)
        g.collect_timings(["enc", "head"])
        g.flush_timings()
        g.record_scalar("loss", 1.0 / (i + 1))
        g.flush(["loss"])
    p = g.profile()
    assert p.source == "host_clock" and len(p.nodes) == len(g.order)
    assert p.timing("enc") > 0 and p.total >= max(n.duration for n in p.nodes)
    split_level = [l for l in p.levels if l.num_nodes == 2]
    assert split_level and split_level[0].parallelism() > 0
    st = g.profile_stats()
    assert st.samples == 3 and st.total_min <= st.total_mean
    assert len(g.timing_trend("enc")) == 3
    assert set(g.timing()) == {n.id for n in p.nodes}
    svg = g.heatmap_svg(str(tmp_path / "h.svg"))
    assert svg.startswith("<svg") and svg.count("<rect") == len(g.order)
    g.plot_html(str(tmp_path / "p.html"))
    g.plot_timings_html(str(tmp_path / "t.html"))
    g.export_trends(str(tmp_path / "tr.csv"))
    g.export_timing_trends(str(tmp_path / "tt.csv"))
    g.write_log(str(tmp_path / "log.txt"), 3)
    assert (tmp_path / "tr.csv").read_text().splitlines()[0] == "flush,loss"
    assert (tmp_path / "log.txt").read_text().splitlines()[2].startswith("epoch 3/3 loss=0.3333")
    assert "enc" in (tmp_path / "t.html").read_text()
    g.disable_profiling()
    n = len(g.profiler.samples)
    g(x)
    assert len(g.profiler.samples) == n


def test_snapshot_cpu_background_save(tmp_path):
    from flodl_b200.nn.checkpoint import load_checkpoint
    g = FlowBuilder.from_(Linear(4, 4)).through(LayerNorm(4)).build()
    snap = g.snapshot_cpu()
    before = [t.clone() for _, t in snap.named]
    with torch.no_grad():
        for p in g.parameters():
            p.add_(1.0)  # training continues; the snapshot is unaffected
    snap.save_background(str(tmp_path / "m.fdl")).join()
    g2 = FlowBuilder.from_(Linear(4, 4)).through(LayerNorm(4)).build()
    rep = load_checkpoint(str(tmp_path / "m.fdl"), g2.graph_named_parameters(), (), g2.structural_hash())
    for (_, t), ref in zip(g2.graph_named_parameters(), before):
        torch.testing.assert_close(t.detach(), ref)


def test_training_glue_with_data_loader():
    from flodl_b200.data import DataLoader, TensorDataSet
    from flodl_b200.optim import SGD, StepDecay
    g = FlowBuilder.from_(Linear(3, 1)).build()
    x = torch.randn(64, 3)
    dl = DataLoader.from_dataset(TensorDataSet(x, x.sum(1, keepdim=True))).batch_size(16).build()
    g.set_data_loader(dl)
    g.set_optimizer(SGD(g.parameters(), lr=0.1))
    g.set_scheduler(StepDecay(0.1, 2, 0.5))
    first = last = None
    for ep in range(6):
        for xb, yb in g.epoch_batches(ep):
            loss = torch.nn.functional.mse_loss(g(xb), yb)
            loss.backward()
            g.step()
            first = first if first is not None else loss.item()
            last = loss.item()
    assert last < first and g.step_count() == 24
