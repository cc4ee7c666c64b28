"""Model zoo (reference ddp-bench models) and the DDP bench harness, on CPU."""
import warnings

import pytest
import torch

from flodl_b200.models.zoo import ZOO


@pytest.mark.parametrize("name", [n for n in ZOO if n != "olmo"])
def test_zoo_model_trains_one_step(name):
    warnings.filterwarnings("ignore")
    spec = ZOO[name]
    torch.manual_seed(0)
    m = spec.build(None)
    ds = spec.dataset(16)
    batch = [t[:4] for t in ds.tensors]
    opt = spec.optimizer(m.parameters(), spec.lr)
    l0 = spec.train_fn(m, batch)
    l0.backward()
    opt.step()
    opt.zero_grad()
    l1 = spec.train_fn(m, batch)
    assert torch.isfinite(l0) and torch.isfinite(l1)
    assert float(l1.detach()) < float(l0.detach()) + 1e-3


def test_olmo_150m_shape():
    from flodl_b200.models.zoo import OLMo
    with torch.device("meta"):
        m = OLMo(device="meta")
    n = sum(p.numel() for p in m.parameters())
    assert 185e6 < n < 195e6  # 150M non-embedding + untied 50304x768 embedding and head


def test_ddp_bench_harness_two_cpu_ranks():
    from flodl_b200.ddp_bench import run
    r = run("mlp", "cpu-cadence", ["cpu", "cpu"], epochs=2, batch_size=32, dataset_size=256)
    assert r["final_loss"] is not None and r["samples_per_s"] > 0
    assert r["syncs"] > 0


def test_ddp_report_tables_elche_and_charts(tmp_path):
    from flodl_b200.ddp_report import bar_chart_svg, line_chart_svg, write_report
    rs = [{"model": "mlp", "mode": "solo", "devices": ["cpu"], "wall_s": 2.0, "samples_per_s": 500.0,
           "first_loss": 2.3, "final_loss": 0.4, "syncs": 0, "batch_counts": []},
          {"model": "mlp", "mode": "nccl-cadence", "devices": ["cpu", "cpu"], "wall_s": 1.2,
           "samples_per_s": 830.0, "first_loss": 2.3, "final_loss": 0.5, "syncs": 6,
           "batch_counts": [[4, 4], [5, 3], [6, 4]]}]
    text = write_report(rs, str(tmp_path / "r.md"), str(tmp_path / "charts"))
    assert "| nccl-cadence | 2 | 1.2 | 830 | 1.66 |" in text
    assert "anchor sequence [4, 5, 6]" in text and "r1 3-4" in text
    assert (tmp_path / "charts" / "mlp-throughput.svg").read_text().startswith("<svg")
    assert "polyline" in line_chart_svg({"a": [1.0, 0.5, 0.2]}, "loss")
    assert bar_chart_svg({"x": 1.0}, "t").count("<rect") == 1
