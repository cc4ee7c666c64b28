"""DistilBERT fine-tuning through the managed and cooperative training tiers
(reference: hf-ddp/src/main.rs). Synthetic token data with a learnable rule
(label = whether token 5 appears) stands in for a text dataset; the model is a
randomly initialised DistilBERT-shaped classifier (no network here; point
``AutoModelForSequenceClassification.from_pretrained`` at a local directory
for real weights).

    python -m flodl_b200.examples.hf_ddp [--tier managed|cooperative] [--cpu-ranks 2]
"""
from __future__ import annotations

import argparse

import torch
import torch.nn.functional as F

from flodl_b200.data import TensorDataSet
from flodl_b200.models.encoders import DistilBertConfig, DistilBertForSequenceClassification
from flodl_b200.optim import AdamW
from flodl_b200.parallel.config import ElCheMode, TrainerConfig
from flodl_b200.parallel.trainer import Trainer

CFG = dict(vocab_size=64, dim=32, n_layers=2, n_heads=2, hidden_dim=64, max_position_embeddings=32,
           num_labels=2)


def make_model(device):
    torch.manual_seed(0)
    return DistilBertForSequenceClassification(DistilBertConfig(**CFG), device=device)


def make_opt(params):
    return AdamW(params, lr=2e-3, weight_decay=0.01)


def train_step(model, batch):
    ids, mask, y = batch
    return F.cross_entropy(model(ids, mask).float(), y)


def dataset(n=512, seq=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(6, 64, (n, seq), generator=g)
    pos = torch.randint(0, n, (n // 2,), generator=g)
    ids[pos, torch.randint(1, seq, (n // 2,), generator=g)] = 5
    ids[:, 0] = 1  # [CLS]-like
    mask = torch.ones_like(ids)
    y = (ids == 5).any(1).long()
    return TensorDataSet(ids, mask, y)


def run(tier: str = "managed", cpu_ranks: int = 0, epochs: int = 4) -> dict:
    cfg = TrainerConfig().batch_size(32).num_epochs(epochs)
    b = Trainer.builder(make_model, make_opt, train_step).dataset(dataset()).config(cfg)
    if tier == "cooperative":
        w = b.mode(ElCheMode.NcclSync).into_worker(rank=0, world=1)
        while (plan := w.next_plan()) is not None:
            for batch in plan:
                w.step(train_step(w.model, batch))
            w.sync()
        st = w.finish()
        return {"tier": tier, "world": 1, "first": st.losses[0], "last": sum(st.losses[-8:]) / 8}
    if cpu_ranks:
        b = b.devices(["cpu"] * cpu_ranks)
    st = b.run().join()
    return {"tier": tier, "world": st.world, "first": st.losses[0], "last": st.losses[-1]}


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--tier", default="managed", choices=["managed", "cooperative"])
    ap.add_argument("--cpu-ranks", type=int, default=0)
    a = ap.parse_args()
    print(run(a.tier, a.cpu_ranks))
