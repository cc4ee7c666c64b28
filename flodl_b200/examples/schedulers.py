"""Learning-rate schedules (reference: flodl/examples/schedulers): warmup for
10 epochs then cosine annealing, with a plateau scheduler as secondary
control - the learning rate used is the minimum of the two.

    python -m flodl_b200.examples.schedulers
"""
from __future__ import annotations

import torch

from flodl_b200.nn import GELU, Linear, mse_loss
from flodl_b200.graph import FlowBuilder
from flodl_b200.optim import Adam, CosineScheduler, PlateauScheduler, WarmupScheduler


def run(epochs: int = 100, seed: int = 0) -> dict:
    torch.manual_seed(seed)
    model = FlowBuilder.from_(Linear(4, 32)).through(GELU()).through(Linear(32, 1)).build()
    opt = Adam(model.parameters(), lr=1e-3)
    sched = WarmupScheduler(CosineScheduler(1e-3, 1e-5, epochs - 10), 1e-3, 10)
    plateau = PlateauScheduler(1e-3, 10, 0.5, 1e-6)
    x = torch.randn(256, 4)
    y = x.prod(1, keepdim=True)
    lrs, losses = [], []
    for epoch in range(epochs):
        lr = min(sched.lr(epoch), plateau.lr())
        opt.set_lr(lr)
        loss = mse_loss(model(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
        plateau.observe(loss.item())
        lrs.append(lr)
        losses.append(loss.item())
    return {"lr_warmup_end": lrs[9], "lr_peak": max(lrs), "lr_final": lrs[-1],
            "first_loss": losses[0], "final_loss": losses[-1]}


if __name__ == "__main__":
    print(run())
