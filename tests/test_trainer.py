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
