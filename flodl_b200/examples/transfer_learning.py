"""Transfer learning with graph trees: pretrain an encoder subgraph, save it,
load it into a new model by label path, freeze it and train only the new head
(reference: flodl/examples/transfer_learning, graph/tree.rs).

    python -m flodl_b200.examples.transfer_learning
"""
from __future__ import annotations

import os
import tempfile

import torch

from flodl_b200.graph import FlowBuilder
from flodl_b200.nn import GELU, Linear, cross_entropy_loss, mse_loss, save_checkpoint
from flodl_b200.optim import Adam


def encoder():
    return (FlowBuilder.from_(Linear(8, 32)).tag("proj").through(GELU()).through(Linear(32, 16))
            .label("encoder").build())


def run(steps: int = 200, seed: int = 0) -> dict:
    torch.manual_seed(seed)
    x = torch.randn(512, 8)
    # stage 1: pretrain encoder + reconstruction head
    pre = FlowBuilder.from_(encoder()).through(Linear(16, 8)).build()
    opt = Adam(pre.parameters(), lr=3e-3)
    for _ in range(steps):
        loss = mse_loss(pre(x), x)
        loss.backward()
        opt.step()
        opt.zero_grad()
    enc = pre.child_graph("encoder")
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "encoder.fdl")
        save_checkpoint(path, enc.graph_named_parameters(), enc.graph_named_buffers(),
                        enc.structural_hash())
        # stage 2: new classifier on the pretrained, frozen encoder
        clf = FlowBuilder.from_(encoder()).through(Linear(16, 3)).tag("head").build()
        report = clf.load_subgraph_checkpoint("encoder", path)
    clf.freeze("encoder")
    frozen = [p.detach().clone() for p in clf.parameters_at("encoder")]
    y = (x[:, 0] > 0).long() + (x[:, 1] > 0).long()
    opt = Adam([p for p in clf.parameters() if p.requires_grad], lr=1e-2)
    first = None
    for _ in range(steps):
        loss = cross_entropy_loss(clf(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
        first = loss.item() if first is None else first
    unchanged = all(torch.equal(a, b) for a, b in zip(frozen, clf.parameters_at("encoder")))
    acc = float((clf(x).argmax(-1) == y).float().mean())
    return {"loaded": len(report.loaded), "first_loss": first, "final_loss": loss.item(),
            "encoder_unchanged": unchanged, "accuracy": acc}


if __name__ == "__main__":
    print(run())
