"""Fit y = sin(x) on [-pi, pi] with a FlowBuilder MLP and a warmup+cosine
learning-rate schedule (reference: flodl/examples/sine_wave).

    python -m flodl_b200.examples.sine_wave [--steps 600]
"""
from __future__ import annotations

import argparse
import math

import torch

from flodl_b200.graph import FlowBuilder
from flodl_b200.nn import Linear, Tanh, mse_loss
from flodl_b200.optim import Adam, CosineScheduler, WarmupScheduler


def run(steps: int = 600, seed: int = 0) -> dict:
    torch.manual_seed(seed)
    model = (FlowBuilder.from_(Linear(1, 32)).through(Tanh()).through(Linear(32, 32))
             .through(Tanh()).through(Linear(32, 1)).build())
    opt = Adam(model.parameters(), lr=1e-2)
    sched = WarmupScheduler(CosineScheduler(1e-2, 1e-4, steps), 1e-2, steps // 10)
    x = torch.linspace(-math.pi, math.pi, 256)[:, None]
    y = torch.sin(x)
    first = None
    for step in range(steps):
        opt.set_lr(sched.lr(step))
        loss = mse_loss(model(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
        first = loss.item() if first is None else first
    with torch.no_grad():
        final = float(mse_loss(model(x), y))
    return {"first_loss": first, "final_loss": final, "final_lr": sched.lr(steps - 1)}


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=600)
    print(run(ap.parse_args().steps))
