"""Embedding, GELU, conv and batch-norm entry points of the op layer."""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from ._common import C, grad_buffer, grad_ready, use_kernels, wants_grad


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight):
        ids_c = ids.reshape(-1).to(torch.int64).contiguous()
        V, Cd = weight.shape
        out = torch.empty((ids_c.numel(), Cd), device=ids.device, dtype=torch.float32)
        C().embed_fwd(ids_c, weight.detach(), None, None, None, out, None, 1)
        ctx.save_for_backward(ids_c, weight)
        return out.reshape(*ids.shape, Cd)

    @staticmethod
    def backward(ctx, dy):
        ids_c, weight = ctx.saved_tensors
        if wants_grad(weight):
            g = grad_buffer(weight)
            C().embed_bwd_atomic(ids_c, dy.reshape(-1, weight.shape[1]).float().contiguous(), g)
            grad_ready(weight)
        return None, None


def embedding(ids: torch.Tensor, weight: torch.Tensor, padding_idx: Optional[int] = None) -> torch.Tensor:
    """Row gather ``weight[ids]`` (f32 table). Gradient rows of ``padding_idx``
    stay zero, as in floDl."""
    if not use_kernels(weight) or weight.dtype != torch.float32 or weight.shape[1] % 4 or padding_idx is not None:
        return F.embedding(ids, weight, padding_idx=padding_idx)
    return _EmbeddingFn.apply(ids, weight)


class _GeluFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        xc = x.contiguous()
        y = torch.empty_like(xc)
        C().gelu_fwd(xc, y)
        ctx.save_for_backward(xc)
        return y

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        dx = torch.empty_like(x)
        C().gelu_bwd(dy.contiguous().to(torch.bfloat16), x, dx)
        return dx


def gelu(x: torch.Tensor) -> torch.Tensor:
    """Exact (erf) GELU; bf16 CUDA tensors run the sm_100a kernel."""
    if use_kernels(x) and x.dtype == torch.bfloat16:
        return _GeluFn.apply(x)
    return F.gelu(x)


def conv2d(x, weight, bias=None, stride=1, padding=0, dilation=1, groups=1):
    return F.conv2d(x, weight, bias, stride, padding, dilation, groups)


def batch_norm2d(x, running_mean, running_var, weight, bias, training, momentum, eps):
    return F.batch_norm(x, running_mean, running_var, weight, bias, training, momentum, eps)
