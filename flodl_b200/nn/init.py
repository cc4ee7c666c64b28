"""Weight initialisers (flodl/src/nn/init.rs)."""
from __future__ import annotations

import math
from typing import Sequence

import torch


def _t(shape, device):
    return torch.empty(tuple(shape), device=device, dtype=torch.float32)


def kaiming_uniform(shape: Sequence[int], fan_in: int, a: float = 0.0, device="cpu") -> torch.Tensor:
    gain = math.sqrt(2.0 / (1.0 + a * a))
    bound = gain * math.sqrt(3.0 / fan_in)
    return _t(shape, device).uniform_(-bound, bound)


def kaiming_normal(shape: Sequence[int], fan_in: int, a: float = 0.0, device="cpu") -> torch.Tensor:
    gain = math.sqrt(2.0 / (1.0 + a * a))
    return _t(shape, device).normal_(0.0, gain / math.sqrt(fan_in))


def xavier_uniform(shape: Sequence[int], fan_in: int, fan_out: int, device="cpu") -> torch.Tensor:
    bound = math.sqrt(6.0 / (fan_in + fan_out))
    return _t(shape, device).uniform_(-bound, bound)


def xavier_normal(shape: Sequence[int], fan_in: int, fan_out: int, device="cpu") -> torch.Tensor:
    return _t(shape, device).normal_(0.0, math.sqrt(2.0 / (fan_in + fan_out)))


def uniform_bias(fan_in: int, shape: Sequence[int], device="cpu") -> torch.Tensor:
    bound = 1.0 / math.sqrt(fan_in) if fan_in > 0 else 0.0
    return _t(shape, device).uniform_(-bound, bound)


def uniform(shape: Sequence[int], low: float, high: float, device="cpu") -> torch.Tensor:
    return _t(shape, device).uniform_(low, high)


def normal(shape: Sequence[int], mean: float = 0.0, std: float = 1.0, device="cpu") -> torch.Tensor:
    return _t(shape, device).normal_(mean, std)


def trunc_normal(shape: Sequence[int], mean: float = 0.0, std: float = 1.0, a: float = -2.0,
                 b: float = 2.0, device="cpu") -> torch.Tensor:
    t = _t(shape, device)
    torch.nn.init.trunc_normal_(t, mean, std, a, b)
    return t


def orthogonal(shape: Sequence[int], gain: float = 1.0, device="cpu") -> torch.Tensor:
    t = _t(shape, device)
    torch.nn.init.orthogonal_(t, gain)
    return t
