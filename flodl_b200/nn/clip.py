"""Gradient clipping (flodl/src/nn/clip.rs). ``clip_grad_norm`` on CUDA params
held in an arena runs two sm_100a kernels (sum of squares, coefficient) and
feeds the coefficient to the fused optimizer as a device scalar, with no host
synchronisation."""
from __future__ import annotations

from typing import Iterable, Optional

import torch

from .._ext import cuda_ext


@torch.no_grad()
def clip_grad_norm(params: Iterable[torch.Tensor], max_norm: float,
                   optimizer=None) -> torch.Tensor:
    """Scale gradients so their global L2 norm is at most ``max_norm``.

    Returns the pre-clip norm as a 0-d tensor. With ``optimizer`` given and its
    groups in arenas, the scale is applied inside the fused optimizer step.
    """
    params = [p for p in params if p.grad is not None]
    if not params:
        return torch.zeros(())
    dev = params[0].device
    if dev.type == "cuda" and optimizer is not None and all(
            g.arena is not None and g.arena.is_bound() for g in optimizer.groups):
        C = cuda_ext()
        ss = torch.zeros((), device=dev)
        for g in optimizer.groups:
            C.sumsq(g.arena.grad, ss)
        if optimizer.gscale_t is None:
            optimizer.gscale_t = torch.ones((), device=dev)
        norm = torch.empty((), device=dev)
        C.clip_coef(ss, float(max_norm), optimizer.gscale_t, norm)
        return norm
    norms = torch._foreach_norm([p.grad for p in params])
    total = torch.linalg.vector_norm(torch.stack([n.to(dev) for n in norms]))
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    torch._foreach_mul_([p.grad for p in params], coef)
    return total


@torch.no_grad()
def clip_grad_value(params: Iterable[torch.Tensor], clip_value: float) -> None:
    for p in params:
        if p.grad is not None:
            p.grad.clamp_(-clip_value, clip_value)
