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
