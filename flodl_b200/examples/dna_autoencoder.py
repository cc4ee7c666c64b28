"""DNA-sequence convolutional autoencoder (reference: flodl/examples/bio/
dna_autoencoder). One-hot [B, 4, L] -> encoder (Conv1d x2 + pooling ->
Linear, tagged "latent") -> decoder (Linear -> ConvTranspose1d x2) -> logits
[B, 4, L]; argmax over bases reconstructs the sequence. Encoder and decoder
are separate graphs with their own checkpoints; ``embed`` returns latents.

    python -m flodl_b200.examples.dna_autoencoder [--epochs 30]
"""
from __future__ import annotations

import argparse
import os
import tempfile

import torch
import torch.nn.functional as F

from flodl_b200.graph import FlowBuilder
from flodl_b200.nn import (Conv1d, ConvTranspose1d, Flatten, Linear, MaxPool1d, ReLU,
                           load_checkpoint, save_checkpoint)
from flodl_b200.nn.module import Module
from flodl_b200.optim import Adam

BASES = "ACGT"


class Unflatten(Module):
    NAME = "unflatten"

    def __init__(self, c, l):
        super().__init__()
        self.c, self.l = c, l

    def forward(self, x):
        return x.view(x.shape[0], self.c, self.l)


class DnaAutoencoder:
    def __init__(self, seq_len: int, latent_dim: int):
        self.L, self.latent = seq_len, latent_dim
        flat = 64 * (seq_len // 4)
        self.encoder = (FlowBuilder.from_(Conv1d(4, 32, 5, padding=2)).through(ReLU()).through(MaxPool1d(2))
                        .through(Conv1d(32, 64, 5, padding=2)).through(ReLU()).through(MaxPool1d(2))
                        .through(Flatten()).through(Linear(flat, latent_dim)).tag("latent").build())
        self.decoder = (FlowBuilder.from_(Linear(latent_dim, flat)).through(ReLU())
                        .through(Unflatten(64, seq_len // 4))
                        .through(ConvTranspose1d(64, 32, 2, stride=2)).through(ReLU())
                        .through(ConvTranspose1d(32, 4, 2, stride=2)).build())

    def parameters(self):
        return list(self.encoder.parameters()) + list(self.decoder.parameters())

    def forward(self, x):
        return self.decoder(self.encoder(x))

    def embed(self, x):
        with torch.no_grad():
            return self.encoder(x)

    def predict(self, x):
        with torch.no_grad():
            idx = self.forward(x).argmax(1)
        return ["".join(BASES[i] for i in row) for row in idx.tolist()]

    def save(self, d):
        for name, g in (("encoder", self.encoder), ("decoder", self.decoder)):
            save_checkpoint(os.path.join(d, f"{name}.fdl"), g.graph_named_parameters(),
                            g.graph_named_buffers(), g.structural_hash())

    def load(self, d):
        for name, g in (("encoder", self.encoder), ("decoder", self.decoder)):
            load_checkpoint(os.path.join(d, f"{name}.fdl"), g.graph_named_parameters(),
                            g.graph_named_buffers(), g.structural_hash())


def run(epochs: int = 30, n: int = 512, L: int = 64, latent: int = 32, seed: int = 42) -> dict:
    torch.manual_seed(seed)
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, 4, (n, L), generator=g)
    x = F.one_hot(idx, 4).transpose(1, 2).float()
    model = DnaAutoencoder(L, latent)
    opt = Adam(model.parameters(), lr=3e-3)
    for _ in range(epochs):
        for i in range(0, n, 64):
            loss = F.cross_entropy(model.forward(x[i:i + 64]), idx[i:i + 64])
            loss.backward()
            opt.step()
            opt.zero_grad()
    orig = ["".join(BASES[i] for i in row) for row in idx[:64].tolist()]
    rec = model.predict(x[:64])
    acc = sum(a == b for o, r in zip(orig, rec) for a, b in zip(o, r)) / (64 * L)
    with tempfile.TemporaryDirectory() as d:
        model.save(d)
        other = DnaAutoencoder(L, latent)
        other.load(d)
        same = other.predict(x[:8]) == rec[:8]
    return {"per_base_accuracy": acc, "reload_matches": same, "latent_shape": list(model.embed(x[:2]).shape)}


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--epochs", type=int, default=30)
    print(run(ap.parse_args().epochs))
