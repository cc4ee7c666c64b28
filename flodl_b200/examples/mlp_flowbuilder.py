"""Quickstart: a FlowBuilder MLP regression trained on the CPU.

BASELINE config 1 and the reference's README example (README.md:79-89,
flodl/examples/quickstart): ``Linear(2,16) -> GELU -> LayerNorm(16) ->
Linear(16,2)`` built with :class:`FlowBuilder`, MSE loss, Adam lr 1e-3, 1000
steps on batches of 256 with ``x ~ N(0, 1)`` and ``y = x A + 0.01 N(0, 1)``
for a fixed seeded 2x2 map ``A``. Runs in a single process without a GPU.

    python -m flodl_b200.examples.mlp_flowbuilder [--steps 1000] [--json]
"""
from __future__ import annotations

import argparse
import json
import time

import torch

from flodl_b200.graph import FlowBuilder
from flodl_b200.nn import GELU, LayerNorm, Linear, mse_loss
from flodl_b200.optim import Adam


def build_model():
    return (FlowBuilder.from_(Linear(2, 16)).through(GELU()).through(LayerNorm(16))
            .through(Linear(16, 2)).build())


def run(steps: int = 1000, batch: int = 256, seed: int = 0):
    torch.manual_seed(seed)
    model = build_model()
    opt = Adam(model.parameters(), lr=1e-3)
    g = torch.Generator().manual_seed(seed + 1)
    A = torch.randn(2, 2, generator=g)
    losses = []
    t0 = time.perf_counter()
    for _ in range(steps):
        x = torch.randn(batch, 2, generator=g)
        y = x @ A + 0.01 * torch.randn(batch, 2, generator=g)
        loss = mse_loss(model(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
        losses.append(float(loss.detach()))
    dt = time.perf_counter() - t0
    return {"steps": steps, "first_loss": losses[0], "final_loss": sum(losses[-20:]) / 20,
            "seconds": dt, "steps_per_s": steps / dt, "samples_per_s": steps * batch / dt}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    r = run(a.steps)
    if a.json:
        print(json.dumps(r))
    else:
        print(f"loss {r['first_loss']:.4f} -> {r['final_loss']:.5f} in {r['seconds']:.2f} s "
              f"({r['steps_per_s']:.0f} steps/s)")


if __name__ == "__main__":
    main()
