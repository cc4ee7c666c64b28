"""Linear and logistic regression from first principles (reference:
flodl/examples/regression): ``Linear(1, 1)`` + MSE recovers y = 2x + 1;
``Linear(2, 1)`` + BCE-with-logits separates two Gaussian blobs.

    python -m flodl_b200.examples.regression
"""
from __future__ import annotations

import torch

from flodl_b200.nn import Linear, bce_with_logits_loss, mse_loss
from flodl_b200.optim import SGD


def run(steps: int = 400, seed: int = 0) -> dict:
    torch.manual_seed(seed)
    x = torch.linspace(-1, 1, 128)[:, None]
    y = 2 * x + 1 + 0.01 * torch.randn_like(x)
    lin = Linear(1, 1)
    opt = SGD(lin.parameters(), lr=0.1)
    for _ in range(steps):
        loss = mse_loss(lin(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
    w, b = float(lin.weight), float(lin.bias)
    pts = torch.cat([torch.randn(200, 2) + 2, torch.randn(200, 2) - 2])
    lab = torch.cat([torch.ones(200, 1), torch.zeros(200, 1)])
    logit = Linear(2, 1)
    opt = SGD(logit.parameters(), lr=0.1)
    for _ in range(steps):
        loss = bce_with_logits_loss(logit(pts), lab)
        loss.backward()
        opt.step()
        opt.zero_grad()
    acc = float(((logit(pts) > 0).float() == lab).float().mean())
    return {"slope": w, "intercept": b, "logistic_accuracy": acc}


if __name__ == "__main__":
    print(run())
