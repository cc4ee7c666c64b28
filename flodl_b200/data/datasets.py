"""Built-in datasets (flodl/src/data/datasets/*.rs): MNIST and CIFAR-10 from
their standard binary files, a character-level Shakespeare LM dataset,
NumPy token shards, and synthetic datasets for benchmarks (no network access
is assumed: files are read from a local directory)."""
from __future__ import annotations

import gzip
import os
import struct
from typing import List, Optional

import numpy as np
import torch

from .loader import DataSet, TensorDataSet


def _read_idx(path: str) -> np.ndarray:
    op = gzip.open if path.endswith(".gz") else open
    with op(path, "rb") as f:
        data = f.read()
    magic = struct.unpack(">I", data[:4])[0]
    nd = magic & 0xFF
    shape = struct.unpack(">" + "I" * nd, data[4:4 + 4 * nd])
    return np.frombuffer(data, dtype=np.uint8, offset=4 + 4 * nd).reshape(shape)


def mnist(root: str, train: bool = True) -> TensorDataSet:
    pre = "train" if train else "t10k"
    def find(stem):
        for suf in ("", ".gz"):
            p = os.path.join(root, stem + suf)
            if os.path.exists(p):
                return p
        raise FileNotFoundError(os.path.join(root, stem))
    x = _read_idx(find(f"{pre}-images-idx3-ubyte")).astype(np.float32) / 255.0
    y = _read_idx(find(f"{pre}-labels-idx1-ubyte")).astype(np.int64)
    return TensorDataSet(torch.from_numpy(x).unsqueeze(1), torch.from_numpy(y))


def cifar10(root: str, train: bool = True) -> TensorDataSet:
    files = [f"data_batch_{i}.bin" for i in range(1, 6)] if train else ["test_batch.bin"]
    xs, ys = [], []
    for fn in files:
        raw = np.fromfile(os.path.join(root, fn), dtype=np.uint8).reshape(-1, 3073)
        ys.append(raw[:, 0].astype(np.int64))
        xs.append(raw[:, 1:].reshape(-1, 3, 32, 32).astype(np.float32) / 255.0)
    x = torch.from_numpy(np.concatenate(xs))
    mean = torch.tensor([0.4914, 0.4822, 0.4465]).view(1, 3, 1, 1)
    std = torch.tensor([0.2470, 0.2435, 0.2616]).view(1, 3, 1, 1)
    return TensorDataSet((x - mean) / std, torch.from_numpy(np.concatenate(ys)))


class CharLM(DataSet):
    """Character-level LM windows over a text (e.g. tiny-shakespeare)."""

    def __init__(self, text: str, seq_len: int):
        chars = sorted(set(text))
        self.stoi = {c: i for i, c in enumerate(chars)}
        self.vocab = len(chars)
        self.data = torch.tensor([self.stoi[c] for c in text], dtype=torch.long)
        self.seq = seq_len

    def __len__(self):
        return max(0, len(self.data) - self.seq - 1)

    def get(self, i):
        w = self.data[i:i + self.seq + 1]
        return [w[:-1], w[1:]]


class TokenShards(DataSet):
    """Fixed-length windows over ``.npy`` token shards (OLMo-style)."""

    def __init__(self, paths: List[str], seq_len: int):
        self.arrays = [np.load(p, mmap_mode="r") for p in paths]
        self.seq = seq_len
        self.counts = [max(0, (len(a) - 1) // seq_len) for a in self.arrays]
        self.total = sum(self.counts)

    def __len__(self):
        return self.total

    def get(self, i):
        for a, c in zip(self.arrays, self.counts):
            if i < c:
                w = torch.from_numpy(np.asarray(a[i * self.seq:(i + 1) * self.seq + 1], dtype=np.int64))
                return [w[:-1], w[1:]]
            i -= c
        raise IndexError(i)


def synthetic_tokens(n: int, seq_len: int, vocab: int, seed: int = 0) -> TensorDataSet:
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(0, vocab, (n, seq_len + 1), generator=g)
    return TensorDataSet(x[:, :-1].contiguous(), x[:, 1:].contiguous())


def synthetic_images(n: int, shape=(3, 32, 32), classes: int = 10, seed: int = 0) -> TensorDataSet:
    g = torch.Generator().manual_seed(seed)
    return TensorDataSet(torch.randn((n,) + tuple(shape), generator=g),
                         torch.randint(0, classes, (n,), generator=g))
