"""Graph showcase: a loop with a learned halting condition, a soft gate over
experts, a hard switch and a map over slices, trained end to end and profiled
(reference: flodl/examples/showcase).

    python -m flodl_b200.examples.showcase
"""
from __future__ import annotations

import torch

from flodl_b200.graph import ArgmaxSelector, FlowBuilder, SoftmaxRouter
from flodl_b200.nn import GELU, Linear, mse_loss
from flodl_b200.optim import Adam


def run(steps: int = 100, seed: int = 0) -> dict:
    torch.manual_seed(seed)
    d = 8
    step_fn = FlowBuilder.from_(Linear(d, d)).through(GELU()).build()
    g = (FlowBuilder.from_(Linear(4, d)).tag("in")
         .loop_body(step_fn).for_n(3).tag("refine")
         .gate(SoftmaxRouter(d, 2), [Linear(d, d), Linear(d, d)]).tag("moe")
         .switch(ArgmaxSelector(d, 2), [Linear(d, d), Linear(d, d)])
         .map(Linear(d, d)).each()
         .through(Linear(d, 1)).tag("out").build())
    g.enable_profiling()
    opt = Adam(g.parameters(), lr=3e-3)
    x = torch.randn(128, 4)
    y = x[:, :1] * x[:, 1:2]
    first = None
    for _ in range(steps):
        loss = mse_loss(g(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
        first = loss.item() if first is None else first
    prof = g.profile()
    return {"first_loss": first, "final_loss": loss.item(), "nodes": len(prof.nodes),
            "slowest": max(prof.nodes, key=lambda n: n.duration).id, "svg": len(g.heatmap_svg())}


if __name__ == "__main__":
    print(run())
