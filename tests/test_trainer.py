"""Managed trainer on CPU ranks (gloo): sync/cadence/CPU-backend modes and the
single-device path (reference: ddp_tests.rs, cluster_worker_tests.rs smokes)."""
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


def _dataset():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(256, 4, generator=g)
    w = torch.tensor([[1.0], [-2.0], [0.5], [3.0]])
    return TensorDataSet(x, x @ w)


def _run(mode, world, epochs=4):
    cfg = TrainerConfig().batch_size(16).num_epochs(epochs).elche(ElCheConfig().mode(mode).anchor(2))
    b = Trainer.builder(make_model, make_opt, train_fn).dataset(_dataset()).config(cfg)
    if world > 1:
        b = b.devices(["cpu"] * world)
    else:
        b = b.devices(["cpu"])
    return b.run().join(timeout=300)


def test_single_device_learns():
    st = _run(ElCheMode.NcclSync, 1)
    assert st.losses[-1] < st.losses[0] * 0.5


def test_two_rank_sync_averages_every_step_and_learns():
    st = _run(ElCheMode.NcclSync, 2, epochs=6)
    assert st.world == 2 and st.syncs > 0
    assert st.losses[-1] < st.losses[0] * 0.7


def test_two_rank_cadence_uses_elche_windows():
    st = _run(ElCheMode.NcclCadence, 2, epochs=3)
    assert st.batch_counts, "ElChe produced no batch counts"
    assert st.losses[-1] < st.losses[0]


def test_two_rank_cpu_backend():
    st = _run(ElCheMode.CpuSync, 2, epochs=2)
    assert st.syncs > 0 and st.losses[-1] < st.losses[0]


def _cfg_ckpt(tmp_path, epochs, **kw):
    cfg = (TrainerConfig().batch_size(16).num_epochs(epochs)
           .elche(ElCheConfig().mode(ElCheMode.NcclCadence).anchor(2)))
    cfg.save_path_ = str(tmp_path / "run" / "ckpt")
    cfg.checkpoint_every_ = 1
    for k, v in kw.items():
        setattr(cfg, k, v)
    return cfg


def test_checkpoint_bundle_meta_v5_and_resume(tmp_path):
    import json
    (tmp_path / "run").mkdir()
    cfg = _cfg_ckpt(tmp_path, 2)
    st = Trainer.builder(make_model, make_opt, train_fn).dataset(_dataset()).config(cfg) \
        .devices(["cpu"] * 2).run().join(timeout=300)
    meta = json.loads((tmp_path / "run" / "ckpt.meta.json").read_text())
    assert meta["schema_version"] == 5 and meta["epoch"] == 1 and meta["world_size_at_save"] == 2
    assert meta["save_reason"] == "checkpoint" and meta["global_step"] > 0 and meta["sync_round"] == st.syncs
    es = meta["elche_state"]
    assert es["phase"] in ("probe", "warmup", "stable", "mature") and len(es["smoothed_ms_per_batch"]) == 2
    # resume: epochs 2..3 only
    cfg2 = _cfg_ckpt(tmp_path, 4, resume_from_=str(tmp_path / "run" / "ckpt"))
    st2 = Trainer.builder(make_model, make_opt, train_fn).dataset(_dataset()).config(cfg2) \
        .devices(["cpu"] * 2).run().join(timeout=300)
    assert st2.start_epoch == 2 and len(st2.losses) == 2
    assert st2.losses[-1] < st.losses[0]


def test_bundle_meta_roundtrip_paths_and_death_records(tmp_path):
    import json

    import pytest

    from flodl_b200.parallel.bundle import (CheckpointBundle, CheckpointMeta, CoverageBlock,
                                            ElCheState, EpochCoverage, RankDeathRecord, SaveReason)
    assert CheckpointBundle.meta_path("a/ckpt.fdl") == "a/ckpt.meta.json"
    assert CheckpointBundle.meta_path("a/ckpt") == "a/ckpt.meta.json"
    assert CheckpointBundle.death_record_path("a/ckpt", 3) == "a/ckpt.rank3.death.json"
    m = CheckpointMeta(4, 100, 12, 8, SaveReason.ReduceStall,
                       ElCheState(6, 2, [10.0, 12.5], "mature", 9, [0.1, 0.2]),
                       CoverageBlock(7, 32, [EpochCoverage(4, 1024, [(0, 32), (512, 64)])]))
    d = json.loads(json.dumps(m.to_json()))
    assert d["save_reason"] == "reduce_stall" and d["coverage"]["per_epoch"][0]["uncovered_ranges"] == [[0, 32], [512, 64]]
    back = CheckpointMeta.from_json(d)
    assert back.coverage.per_epoch[0].uncovered_ranges == [(0, 32), (512, 64)] and back.elche_state.anchor == 6
    assert SaveReason.from_u8(SaveReason.Checkpoint.to_u8()) is SaveReason.Checkpoint and SaveReason.from_u8(9) is None
    with pytest.raises(ValueError, match="newer"):
        CheckpointMeta.from_json(dict(d, schema_version=6))
    p = str(tmp_path / "x.rank1.death.json")
    RankDeathRecord(1, 4, "RuntimeError('boom')").write_to_file(p)
    r = RankDeathRecord.read(p)
    assert r.rank == 1 and r.schema_version == 1 and r.unix_time_secs > 0


def test_checkpoint_forge_writes_in_background(tmp_path):
    from flodl_b200.parallel.bundle import CheckpointForge, CheckpointMeta, bundle_complete, load_bundle
    model, opt = make_model("cpu"), None
    forge = CheckpointForge()
    forge.save(str(tmp_path / "f"), model, opt, CheckpointMeta(0, 1, 0, 1))
    forge.join()
    assert bundle_complete(str(tmp_path / "f"))
    assert load_bundle(str(tmp_path / "f"), make_model("cpu")).global_step == 1
