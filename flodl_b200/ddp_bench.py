"""DDP benchmark harness over the model zoo (the reference's ddp-bench).

    python -m flodl_b200.ddp_bench --model mlp [--mode nccl-cadence] [--devices cpu,cpu]
                                   [--epochs 1] [--batches 0] [--batch-size B] [--json]

Runs one model of :data:`flodl_b200.models.zoo.ZOO` through the managed
trainer (``Trainer.builder(...).run()``, one process per device) in one of the
reference's DDP modes - ``solo`` (one device), ``nccl-sync``,
``nccl-cadence`` (ElChe windows), ``cpu-sync``, ``cpu-cadence``,
``cpu-async`` (EASGD blend) - and reports wall time, samples/s, first/final
loss, the number of averaging rounds and ElChe's batch counts as one JSON line.
The device list may mix CUDA devices and ``cpu`` ranks (gloo).
"""
from __future__ import annotations

import argparse
import json
import time

import torch

MODES = {
    "solo": "NcclSync", "nccl-sync": "NcclSync", "nccl-cadence": "NcclCadence",
    "cpu-sync": "CpuSync", "cpu-cadence": "CpuCadence", "cpu-async": "CpuAsync",
}


class _Build:
    """Picklable factory (rank processes are spawned): looks the model up by name."""

    def __init__(self, name):
        self.name = name

    def __call__(self, device):
        from .models.zoo import ZOO
        return ZOO[self.name].build(device)


class _Opt:
    def __init__(self, name, lr):
        self.name, self.lr = name, lr

    def __call__(self, params):
        from .models.zoo import ZOO
        return ZOO[self.name].optimizer(params, self.lr)


class _Train:
    def __init__(self, name):
        self.name = name

    def __call__(self, model, batch):
        from .models.zoo import ZOO
        return ZOO[self.name].train_fn(model, batch)


def run(model: str, mode: str = "nccl-cadence", devices=("cpu",), epochs: int = 1,
        batch_size: int = 0, dataset_size: int = 0, lr: float = 0.0, anchor: int = 4) -> dict:
    from .models.zoo import ZOO
    from .parallel import ElCheConfig, ElCheMode, Trainer, TrainerConfig

    spec = ZOO[model]
    bs = batch_size or spec.batch_size
    ds = spec.dataset(dataset_size) if dataset_size else spec.dataset()
    lr_ = lr or spec.lr
    devs = list(devices) if mode != "solo" else [list(devices)[0]]
    cfg = (TrainerConfig().batch_size(bs).num_epochs(epochs)
           .elche(ElCheConfig().mode(getattr(ElCheMode, MODES[mode])).anchor(anchor)))
    t0 = time.perf_counter()
    st = (Trainer.builder(_Build(model), _Opt(model, lr_), _Train(model))
          .dataset(ds).config(cfg).devices(devs).run().join(timeout=3600))
    dt = time.perf_counter() - t0
    n = len(ds) * epochs
    return {"model": model, "description": spec.description, "mode": mode, "devices": devs,
            "epochs": epochs, "batch_size": bs, "samples": n, "wall_s": round(dt, 3),
            "samples_per_s": round(n / dt, 1),
            "first_loss": st.losses[0] if st.losses else None,
            "final_loss": st.losses[-1] if st.losses else None,
            "syncs": st.syncs, "batch_counts": st.batch_counts}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="mlp")
    ap.add_argument("--mode", default="nccl-cadence", choices=sorted(MODES))
    ap.add_argument("--devices", default="cpu")
    ap.add_argument("--epochs", type=int, default=1)
    ap.add_argument("--batch-size", type=int, default=0)
    ap.add_argument("--dataset-size", type=int, default=0)
    ap.add_argument("--lr", type=float, default=0.0)
    ap.add_argument("--anchor", type=int, default=4)
    a = ap.parse_args()
    r = run(a.model, a.mode, a.devices.split(","), a.epochs, a.batch_size, a.dataset_size, a.lr,
            a.anchor)
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
