"""Residual stacks with FlowBuilder: ``also`` adds a skip branch, ``split`` +
``merge`` runs parallel experts, ``tag`` names blocks (reference:
flodl/examples/flowbuilder_residual).

    python -m flodl_b200.examples.flowbuilder_residual
"""
from __future__ import annotations

import torch

from flodl_b200.graph import FlowBuilder, MergeOp
from flodl_b200.nn import GELU, LayerNorm, Linear, mse_loss
from flodl_b200.optim import Adam


def block(d):
    return FlowBuilder.from_(LayerNorm(d)).through(Linear(d, 4 * d)).through(GELU()).through(Linear(4 * d, d)).build()


def run(steps: int = 200, seed: int = 0) -> dict:
    torch.manual_seed(seed)
    d = 16
    g = (FlowBuilder.from_(Linear(8, d)).tag("stem")
         .also(block(d)).tag("res1")
         .also(block(d)).tag("res2")
         .split([Linear(d, d), Linear(d, d)]).merge(MergeOp.MEAN).tag("experts")
         .through(Linear(d, 1)).build())
    opt = Adam(g.parameters(), lr=3e-3)
    x = torch.randn(256, 8)
    y = (x ** 2).sum(1, keepdim=True)
    first = None
    for _ in range(steps):
        loss = mse_loss(g(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
        first = loss.item() if first is None else first
    return {"first_loss": first, "final_loss": loss.item(), "levels": len(g.levels),
            "tags": g.tag_names_list()}


if __name__ == "__main__":
    print(run())
