"""Mixed precision: bf16 autocast for the forward, f32 master weights, and
dynamic loss scaling with GradScaler (reference: flodl/examples/
mixed_precision). Autocast runs on CUDA when present, else on the CPU.

    python -m flodl_b200.examples.mixed_precision [--steps 300]
"""
from __future__ import annotations

import argparse

import torch

from flodl_b200.graph import FlowBuilder
from flodl_b200.nn import GELU, GradScaler, LayerNorm, Linear, autocast, mse_loss
from flodl_b200.optim import AdamW


def run(steps: int = 300, seed: int = 0) -> dict:
    torch.manual_seed(seed)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    model = (FlowBuilder.from_(Linear(16, 64, device=dev)).through(GELU()).through(LayerNorm(64, device=dev))
             .through(Linear(64, 4, device=dev)).build())
    opt = AdamW(model.parameters(), lr=3e-3, weight_decay=0.01)
    scaler = GradScaler(init_scale=2.0 ** 10)
    A = torch.randn(16, 4, device=dev)
    losses, skipped = [], 0
    for _ in range(steps):
        x = torch.randn(128, 16, device=dev)
        with autocast(torch.bfloat16, device_type=dev):
            out = model(x)
        loss = mse_loss(out.float(), x @ A)
        scaler.scale_loss(loss).backward()
        if not scaler.step(opt):
            skipped += 1
        scaler.update()
        opt.zero_grad()
        losses.append(loss.item())
    return {"first_loss": losses[0], "final_loss": sum(losses[-10:]) / 10, "skipped": skipped,
            "scale": scaler.scale, "weight_dtype": str(list(model.parameters())[0].dtype)}


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=300)
    print(run(ap.parse_args().steps))
