"""The coordinator-driven trainer on 2-4 GPUs: device averaging through the
fused peer-memory kernel, and survivors that re-form after a rank leaves
between windows. NVLS is off and the kernels use plain peer loads; the rank
leaves only after its last collective finished (nothing of it is in flight),
and the survivors learn of it on the host before their next launch."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def make_model(device):
    from flodl_b200.models import ResNet20
    torch.manual_seed(0)
    return ResNet20(device=device)


def make_opt(params):
    from flodl_b200.optim import SGD
    return SGD(params, 0.05, momentum=0.9)


def train_fn(model, batch):
    x, y = batch
    return model.loss(x, y)


def _dataset(n=2048):
    from flodl_b200.data import TensorDataSet
    g = torch.Generator().manual_seed(3)
    return TensorDataSet(torch.randn(n, 3, 32, 32, generator=g),
                         torch.randint(0, 10, (n,), generator=g))


def _run(world, hooks=None, epochs=2):
    from flodl_b200.parallel import ElCheConfig, ElCheMode, Trainer, TrainerConfig
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    cfg = (TrainerConfig().batch_size(64).num_epochs(epochs)
           .elche(ElCheConfig().mode(ElCheMode.NcclCadence).anchor(2)))
    b = (Trainer.builder(make_model, make_opt, train_fn).dataset(_dataset()).config(cfg)
         .devices([f"cuda:{i}" for i in range(world)]).group_timeout(30))
    if hooks:
        b = b.test_hooks(**hooks)
    return b.run().join(timeout=900)


@pytest.mark.parametrize("world", [2, 4])
def test_cadence_on_gpus_through_the_coordinator(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs (have {torch.cuda.device_count()})")
    st = _run(world)
    rec = st.record
    assert rec["syncs"] > 0 and not rec["deaths"]
    assert all(d >= 0.0 for d in rec["divergence"])
    # BatchNorm running statistics are averaged with the parameters
    names = dict(st.buffers)
    assert torch.isfinite(names["bn1.running_mean"] if "bn1.running_mean" in names
                          else next(iter(names.values())).float()).all()


def test_gpu_rank_leaves_between_windows_survivors_continue():
    world = 3 if torch.cuda.device_count() >= 3 else 2
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    st = _run(world, hooks={"leave_after_syncs": {world - 1: 2}}, epochs=2)
    rec = st.record
    assert [d["rank"] for d in rec["deaths"]] == [world - 1]
    assert rec["sessions"] >= 2
    assert rec["epochs"][-1]["alive"] == list(range(world - 1))
