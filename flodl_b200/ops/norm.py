"""Fused LayerNorm on CUDA (one kernel forward, one kernel backward).

Reference: ``autograd::layer_norm`` -> ``at::native_layer_norm``
(flodl/src/autograd/ops.rs:629, flodl-sys/ops_tensor.cpp:580-600).
The backward accumulates ``weight.grad``/``bias.grad`` in the same pass as the
input gradient and notifies the gradient-ready listeners.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from ._common import C, grad_buffer, grad_ready, use_kernels, wants_grad


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps, out_bf16):
        xc = x.contiguous()
        Cdim = xc.shape[-1]
        rows = xc.numel() // Cdim
        mean = torch.empty(rows, device=x.device, dtype=torch.float32)
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        if out_bf16 or x.dtype == torch.bfloat16:
            y = torch.empty(xc.shape, device=x.device, dtype=torch.bfloat16)
            C().ln_fwd(xc, weight.detach() if weight is not None else None,
                       bias.detach() if bias is not None else None, y, None, mean, rstd, eps)
        else:
            y = torch.empty(xc.shape, device=x.device, dtype=torch.float32)
            C().ln_fwd(xc, weight.detach() if weight is not None else None,
                       bias.detach() if bias is not None else None, None, y, mean, rstd, eps)
        ctx.save_for_backward(xc, weight, bias, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        xc, weight, bias, mean, rstd = ctx.saved_tensors
        dy16 = dy.contiguous()
        if dy16.dtype != torch.bfloat16:
            t = torch.empty(dy16.shape, device=dy.device, dtype=torch.bfloat16)
            C().cast_f32_bf16(dy16.float(), t)
            dy16 = t
        dx_f32 = dx_bf16 = None
        if xc.dtype == torch.bfloat16:
            dx_bf16 = torch.empty_like(xc)
            dx = dx_bf16
        else:
            dx_f32 = torch.empty(xc.shape, device=xc.device, dtype=torch.float32)
            dx = dx_f32
        dg = grad_buffer(weight) if wants_grad(weight) else None
        db = grad_buffer(bias) if wants_grad(bias) else None
        C().ln_bwd(dy16, xc, mean, rstd, weight.detach() if weight is not None else None, None,
                   dx_f32, dx_bf16, dg, db, None)
        if dg is not None:
            grad_ready(weight)
        if db is not None:
            grad_ready(bias)
        return dx, None, None, None, None


def layer_norm(x: torch.Tensor, weight: Optional[torch.Tensor], bias: Optional[torch.Tensor],
               eps: float = 1e-5, out_bf16: bool = False) -> torch.Tensor:
    """LayerNorm over the last dimension.

    On CUDA, ``out_bf16=True`` writes the normalised output in bf16 (the operand
    format of the tcgen05 GEMMs) while statistics stay in f32.
    """
    if not use_kernels(x) or x.shape[-1] % 4 != 0 or x.shape[-1] > 2048 or x.dtype not in (
            torch.float32, torch.bfloat16):
        if x.is_cuda:
            raise RuntimeError(
                f"flodl_b200 layer_norm kernel supports f32/bf16 with C%4==0 and C<=2048 "
                f"(got {x.dtype}, C={x.shape[-1]})")
        return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)
    return _LayerNormFn.apply(x, weight, bias, float(eps), bool(out_bf16))


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        xc = x.contiguous()
        rows = xc.numel() // xc.shape[-1]
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        y = torch.empty_like(xc)
        C().rms_fwd(xc, weight.detach() if weight is not None else None, y, rstd, eps)
        ctx.save_for_backward(xc, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        xc, weight, rstd = ctx.saved_tensors
        dyc = dy.contiguous().to(xc.dtype)
        dx = torch.empty_like(xc)
        dw = grad_buffer(weight) if wants_grad(weight) else None
        C().rms_bwd(dyc, xc, weight.detach() if weight is not None else None, rstd, dx, dw)
        if dw is not None:
            grad_ready(weight)
        return dx, None, None


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float = 1e-5) -> torch.Tensor:
    """RMSNorm over the last dimension, ``x / sqrt(mean(x^2) + eps) * weight``
    (flodl/src/nn/rmsnorm.rs:54-62). On CUDA one kernel forward and one
    backward (which also accumulates ``weight.grad``); f32 and bf16 inputs keep
    their dtype, statistics are f32."""
    if not use_kernels(x) or x.dtype not in (torch.float32, torch.bfloat16) or (
            x.shape[-1] > 8192 and wants_grad(weight)):
        xf = x.float() if x.dtype in (torch.float16, torch.bfloat16) else x  # at least f32
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        y = y * weight if weight is not None else y
        return y.to(x.dtype) if x.dtype in (torch.float16, torch.bfloat16) else y
    return _RMSNormFn.apply(x, weight, float(eps))


class _GroupNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, groups, weight, bias, eps):
        xc = x.contiguous()
        n = xc.shape[0] * groups
        mean = torch.empty(n, device=x.device, dtype=torch.float32)
        rstd = torch.empty(n, device=x.device, dtype=torch.float32)
        y = torch.empty_like(xc)
        C().gn_fwd(xc, weight.detach() if weight is not None else None,
                   bias.detach() if bias is not None else None, y, mean, rstd, groups, eps)
        ctx.groups = groups
        ctx.save_for_backward(xc, weight, bias, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        xc, weight, bias, mean, rstd = ctx.saved_tensors
        dx = torch.empty_like(xc)
        dg = grad_buffer(weight) if wants_grad(weight) else None
        db = grad_buffer(bias) if wants_grad(bias) else None
        C().gn_bwd(dy.contiguous().to(xc.dtype), xc, weight.detach() if weight is not None else None,
                   mean, rstd, dx, dg, db, ctx.groups)
        if dg is not None:
            grad_ready(weight)
        if db is not None:
            grad_ready(bias)
        return dx, None, None, None, None


def group_norm(x: torch.Tensor, groups: int, weight: Optional[torch.Tensor] = None,
               bias: Optional[torch.Tensor] = None, eps: float = 1e-5) -> torch.Tensor:
    """GroupNorm over ``x [N, C, *]`` (flodl/src/nn/groupnorm.rs:62-70): one
    kernel forward, one backward that also accumulates the affine gradients,
    on CUDA for f32 and bf16; elsewhere PyTorch's."""
    if (not use_kernels(x) or x.dtype not in (torch.float32, torch.bfloat16) or x.dim() < 2
            or x.shape[1] % groups):
        return F.group_norm(x, groups, weight, bias, eps)
    return _GroupNormFn.apply(x, int(groups), weight, bias, float(eps))
