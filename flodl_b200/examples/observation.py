"""Observation: tag graph values, collect and flush them per epoch, and stop
when the loss trend stalls (reference: flodl/examples/observation,
graph/observe.rs, trend.rs).

    python -m flodl_b200.examples.observation
"""
from __future__ import annotations

import torch

from flodl_b200.graph import FlowBuilder
from flodl_b200.nn import Linear, ReLU, mse_loss
from flodl_b200.optim import Adam


def run(max_epochs: int = 60, seed: int = 0) -> dict:
    torch.manual_seed(seed)
    g = (FlowBuilder.from_(Linear(4, 32)).through(ReLU()).tag("hidden").through(Linear(32, 1))
         .tag("out").build())
    opt = Adam(g.parameters(), lr=1e-2)
    x = torch.randn(256, 4)
    y = x.sum(1, keepdim=True)
    epochs = 0
    for epoch in range(max_epochs):
        for i in range(0, 256, 64):
            loss = mse_loss(g(x[i:i + 64]), y[i:i + 64])
            loss.backward()
            opt.step()
            opt.zero_grad()
            g.collect(["hidden"], "mean")
            g.record_scalar("loss", loss.item())
        g.flush()
        epochs = epoch + 1
        t = g.trend("loss")
        if len(t) >= 8 and t.stalled(8, 1e-3):
            break
    t = g.trend("loss")
    return {"epochs": epochs, "final_loss": t.latest(), "improving": t.improving(0),
            "hidden_mean": g.trend("hidden").latest(), "metrics": dict(g.latest_metrics())}


if __name__ == "__main__":
    print(run())
