"""Activations (flodl/src/nn/activation.rs:12-330)."""
from __future__ import annotations

import enum

import torch
import torch.nn.functional as F

from .. import ops
from .module import Module


class GeluApprox(enum.Enum):
    NONE = "none"
    TANH = "tanh"


class _Act(Module):
    FN = None

    def forward(self, x):
        return type(self).FN(x)


class ReLU(_Act):
    NAME = "relu"
    FN = staticmethod(F.relu)


class Sigmoid(_Act):
    NAME = "sigmoid"
    FN = staticmethod(torch.sigmoid)


class Tanh(_Act):
    NAME = "tanh"
    FN = staticmethod(torch.tanh)


class SiLU(_Act):
    NAME = "silu"
    FN = staticmethod(F.silu)


class Mish(_Act):
    NAME = "mish"
    FN = staticmethod(F.mish)


class SELU(_Act):
    NAME = "selu"
    FN = staticmethod(F.selu)


class Hardswish(_Act):
    NAME = "hardswish"
    FN = staticmethod(F.hardswish)


class Hardsigmoid(_Act):
    NAME = "hardsigmoid"
    FN = staticmethod(F.hardsigmoid)


class GELU(Module):
    """GELU, exact (erf) by default or tanh-approximated. bf16 CUDA tensors run
    the sm_100a elementwise kernel."""

    NAME = "gelu"

    def __init__(self, approximate: GeluApprox = GeluApprox.NONE):
        super().__init__()
        self.approximate = GeluApprox(approximate) if not isinstance(approximate, GeluApprox) else approximate

    @classmethod
    def tanh(cls):
        return cls(GeluApprox.TANH)

    def forward(self, x):
        if self.approximate == GeluApprox.NONE:
            return ops.gelu(x)
        return F.gelu(x, approximate="tanh")


class SwiGLU(Module):
    """Splits the last dim in halves (a, b) and returns silu(a) * b."""

    NAME = "swiglu"

    def forward(self, x):
        a, b = x.chunk(2, dim=-1)
        return F.silu(a) * b


class LeakyReLU(Module):
    NAME = "leaky_relu"

    def __init__(self, negative_slope: float = 0.01):
        super().__init__()
        self.negative_slope = negative_slope

    def forward(self, x):
        return F.leaky_relu(x, self.negative_slope)


class ELU(Module):
    NAME = "elu"

    def __init__(self, alpha: float = 1.0):
        super().__init__()
        self.alpha = alpha

    def forward(self, x):
        return F.elu(x, self.alpha)


class Softplus(Module):
    NAME = "softplus"

    def __init__(self, beta: float = 1.0, threshold: float = 20.0):
        super().__init__()
        self.beta, self.threshold = beta, threshold

    def forward(self, x):
        return F.softplus(x, self.beta, self.threshold)


class Softmax(Module):
    NAME = "softmax"

    def __init__(self, dim: int = -1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return torch.softmax(x, self.dim)


class LogSoftmax(Softmax):
    NAME = "log_softmax"

    def forward(self, x):
        return torch.log_softmax(x, self.dim)


class PReLU(Module):
    NAME = "prelu"

    def __init__(self, num_parameters: int = 1, init: float = 0.25, device=None):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.full((num_parameters,), init, device=device))

    def forward(self, x):
        return F.prelu(x, self.weight)
