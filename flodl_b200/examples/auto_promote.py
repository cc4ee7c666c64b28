"""Auto-promotion: the same ``Trainer`` call trains on one device, or - with
two or more GPUs visible - promotes to one process per GPU with averaged
replicas (reference: flodl/examples/auto_promote, ddp.rs:408-560).
``devices=["cpu", "cpu"]`` runs the multi-process path on gloo ranks.

    python -m flodl_b200.examples.auto_promote [--cpu-ranks 2]
"""
from __future__ import annotations

import argparse

import torch

from flodl_b200.data import TensorDataSet
from flodl_b200.nn import Linear, ReLU, mse_loss
from flodl_b200.nn.module import Module
from flodl_b200.optim import Adam
from flodl_b200.parallel.config import ElCheMode, TrainerConfig
from flodl_b200.parallel.trainer import Trainer


class Regressor(Module):
    NAME = "regressor"

    def __init__(self, device=None):
        super().__init__()
        self.l1, self.act, self.l2 = Linear(8, 32, device=device), ReLU(), Linear(32, 1, device=device)

    def forward(self, x):
        return self.l2(self.act(self.l1(x)))


def make_model(device):
    torch.manual_seed(0)
    return Regressor(device)


def make_opt(params):
    return Adam(params, lr=3e-3)


def train_step(model, batch):
    x, y = batch
    return mse_loss(model(x), y)


def dataset(n=1024, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, 8, generator=g)
    return TensorDataSet(x, x.sum(1, keepdim=True))


def run(cpu_ranks: int = 0, epochs: int = 3, mode: ElCheMode = ElCheMode.NcclCadence) -> dict:
    b = (Trainer.builder(make_model, make_opt, train_step).dataset(dataset())
         .config(TrainerConfig().batch_size(32).num_epochs(epochs)).mode(mode))
    if cpu_ranks:
        b = b.devices(["cpu"] * cpu_ranks)
    st = b.run().join()
    return {"world": st.world, "mode": st.mode, "epoch_losses": st.losses, "syncs": st.syncs}


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--cpu-ranks", type=int, default=0)
    print(run(ap.parse_args().cpu_ranks))
