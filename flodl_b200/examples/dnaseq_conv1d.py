"""DNA-sequence Conv1d classifier: synthetic ChIP-seq-style motif detection
(reference: flodl/examples/bio/dnaseq_conv1d). Sequences of length 200 are
one-hot encoded to [4, L] (A, C, G, T); half carry the motif TGACGTCA at a
random position; a Conv1d/ReLU/MaxPool1d/Linear stack with binary
cross-entropy learns to detect it.

    python -m flodl_b200.examples.dnaseq_conv1d [--epochs 15]
"""
from __future__ import annotations

import argparse

import torch

from flodl_b200.graph import FlowBuilder
from flodl_b200.nn import (Conv1d, Dropout, Flatten, Linear, MaxPool1d, ReLU, Sigmoid,
                           bce_loss)
from flodl_b200.optim import Adam

BASES = "ACGT"
MOTIF = "TGACGTCA"


def one_hot(seqs, L):
    idx = torch.tensor([[BASES.index(c) for c in s[:L]] for s in seqs])
    return torch.nn.functional.one_hot(idx, 4).transpose(1, 2).float()  # [B, 4, L]


def make_data(n, L, g):
    seqs, labels = [], []
    for _ in range(n):
        s = [BASES[i] for i in torch.randint(0, 4, (L,), generator=g).tolist()]
        has = bool(torch.rand((), generator=g) < 0.5)
        if has:
            st = int(torch.randint(0, L - len(MOTIF) + 1, (), generator=g))
            s[st:st + len(MOTIF)] = list(MOTIF)
        seqs.append("".join(s))
        labels.append(float(has))
    return one_hot(seqs, L), torch.tensor(labels)[:, None]


def build_model(L):
    flat = 128 * ((L - 4) // 2 // 2)
    return (FlowBuilder.from_(Conv1d(4, 32, 5)).through(ReLU())
            .through(Conv1d(32, 64, 5, padding=2)).through(ReLU()).through(MaxPool1d(2))
            .through(Conv1d(64, 128, 3, padding=1)).through(ReLU()).through(MaxPool1d(2))
            .through(Flatten()).through(Linear(flat, 64)).through(ReLU()).through(Dropout(0.3))
            .through(Linear(64, 1)).through(Sigmoid()).build())


def run(epochs: int = 15, n_train: int = 4000, n_val: int = 500, L: int = 200, seed: int = 42) -> dict:
    torch.manual_seed(seed)
    g = torch.Generator().manual_seed(seed)
    xtr, ytr = make_data(n_train, L, g)
    xva, yva = make_data(n_val, L, g)
    model = build_model(L)
    opt = Adam(model.parameters(), lr=1e-3)
    for _ in range(epochs):
        model.train()
        perm = torch.randperm(n_train, generator=g)
        for i in range(0, n_train, 64):
            b = perm[i:i + 64]
            loss = bce_loss(model(xtr[b]), ytr[b])
            loss.backward()
            opt.step()
            opt.zero_grad()
    model.eval()
    with torch.no_grad():
        acc = float(((model(xva) > 0.5).float() == yva).float().mean())
    return {"val_accuracy": acc, "final_loss": loss.item()}


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--epochs", type=int, default=15)
    print(run(ap.parse_args().epochs))
