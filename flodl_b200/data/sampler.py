"""Samplers (flodl/src/data/sampler.rs): index orders for an epoch."""
from __future__ import annotations

from typing import List, Sequence

import torch


class Sampler:
    def indices(self, epoch: int, n: int) -> List[int]:  # pragma: no cover - interface
        raise NotImplementedError


class SequentialSampler(Sampler):
    def indices(self, epoch, n):
        return list(range(n))


class RandomSampler(Sampler):
    def __init__(self, seed: int = 0):
        self.seed = seed

    def indices(self, epoch, n):
        g = torch.Generator()
        g.manual_seed(self.seed * 1000003 + epoch)
        return torch.randperm(n, generator=g).tolist()


class DistributedSampler(Sampler):
    """Rank ``rank`` of ``world`` takes every ``world``-th index of a shared
    per-epoch permutation (padded so ranks get equal counts)."""

    def __init__(self, rank: int, world: int, seed: int = 0, shuffle: bool = True):
        self.rank, self.world, self.seed, self.shuffle = rank, world, seed, shuffle

    def indices(self, epoch, n):
        base = RandomSampler(self.seed).indices(epoch, n) if self.shuffle else list(range(n))
        per = (n + self.world - 1) // self.world
        base = base + base[: per * self.world - n]
        return base[self.rank::self.world]


class ChunkSampler(Sampler):
    """Serve an explicit list of index ranges (the ElChe progressive chunk pool
    hands each rank ranges of the epoch permutation)."""

    def __init__(self, ranges: Sequence[tuple], seed: int = 0):
        self.ranges, self.seed = list(ranges), seed

    def indices(self, epoch, n):
        perm = RandomSampler(self.seed).indices(epoch, n)
        out = []
        for a, b in self.ranges:
            out.extend(perm[a:b])
        return out
