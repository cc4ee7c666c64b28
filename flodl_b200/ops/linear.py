"""Fused Linear: ``y = act(x W^T + b) [+ residual]`` on the tcgen05 GEMM engine.

Reference: ``autograd::linear`` -> ``torch::linear`` (flodl/src/autograd/ops.rs:576,
flodl-sys/ops_training.cpp:400-414). On CUDA the forward is one GEMM whose
epilogue adds the bias, applies GELU (keeping the pre-activation for backward)
and adds the residual; backward is two GEMMs (dgrad with the GELU derivative in
its epilogue, split-K wgrad accumulating into ``weight.grad``) plus the bias
column sum.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from ._common import (C, as_bf16_2d, bf16_shadow, grad_buffer, grad_ready, splitk_for,
                      use_kernels, wants_grad)


def gelu_op(y):
    from .misc import gelu
    return gelu(y)


def wgrad_accumulate(dy2: torch.Tensor, x2: torch.Tensor, weight: torch.Tensor,
                     alpha_t: Optional[torch.Tensor] = None) -> None:
    """weight.grad += dy2^T @ x2  (dy2 [T, N] bf16, x2 [T, K] bf16)."""
    T, N = dy2.shape
    K = x2.shape[1]
    g = grad_buffer(weight)
    ks = splitk_for(N, K, T)
    C().gemm(dy2, x2, g, N, K, T, True, True, flags=C().EPI_ACCUMULATE, k_splits=ks,
             alpha_t=alpha_t)


def bias_grad_accumulate(dy2: torch.Tensor, bias: torch.Tensor) -> None:
    C().colsum(dy2, grad_buffer(bias))


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, act, residual):
        K = x.shape[-1]
        N = weight.shape[0]
        x2 = as_bf16_2d(x)
        T = x2.shape[0]
        w16 = bf16_shadow(weight)
        out_f32 = residual is not None
        out = torch.empty((T, N), device=x.device,
                          dtype=torch.float32 if out_f32 else torch.bfloat16)
        flags = 0
        aux = None
        if act == "gelu":
            flags |= C().EPI_GELU
            aux = torch.empty((T, N), device=x.device, dtype=torch.bfloat16)
        res2 = residual.reshape(T, N).float().contiguous() if residual is not None else None
        C().gemm(x2, w16, out, T, N, K, False, False, bias=bias.detach() if bias is not None else None,
                 residual=res2, aux=aux, flags=flags)
        ctx.save_for_backward(x2, weight, bias, aux)
        ctx.act = act
        ctx.x_shape = x.shape
        ctx.x_dtype = x.dtype
        ctx.has_res = residual is not None
        return out.reshape(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, bias, aux = ctx.saved_tensors
        N, K = weight.shape
        dy2 = as_bf16_2d(dy)
        T = dy2.shape[0]
        if ctx.act == "gelu":
            # dy of the pre-activation: dy * GELU' (kept by the forward epilogue)
            dh = torch.empty((T, N), device=dy.device, dtype=torch.bfloat16)
            C().mul_bf16(dy2.contiguous(), aux, dh)
            dy2 = dh
        dx = None
        if ctx.needs_input_grad[0]:
            w16 = bf16_shadow(weight)
            out_dtype = torch.float32 if ctx.x_dtype == torch.float32 else torch.bfloat16
            dx2 = torch.empty((T, K), device=dy.device, dtype=out_dtype)
            C().gemm(dy2, w16, dx2, T, K, N, False, True)
            dx = dx2.reshape(ctx.x_shape)
        if wants_grad(weight):
            wgrad_accumulate(dy2, x2, weight)
            grad_ready(weight)
        if bias is not None and wants_grad(bias):
            bias_grad_accumulate(dy2, bias)
            grad_ready(bias)
        dres = dy if ctx.has_res else None
        return dx, None, None, None, dres


class _SmallLinearFn(torch.autograd.Function):
    """Forward and input gradient on the library GEMM (bf16 operands from the
    cached weight shadow, f32 accumulation); the weight and bias gradients
    accumulate into ``.grad`` through the split-K tcgen05 GEMM and fire the
    gradient-ready listeners, exactly as the fused path does."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        x2 = as_bf16_2d(x)
        w16 = bf16_shadow(weight)
        b16 = bf16_shadow(bias) if bias is not None else None
        out = F.linear(x2, w16, b16)
        ctx.save_for_backward(x2, weight, bias)
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        return out.reshape(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, weight, bias = ctx.saved_tensors
        dy2 = as_bf16_2d(dy)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.mm(dy2, bf16_shadow(weight)).reshape(ctx.x_shape)
            if ctx.x_dtype == torch.float32:
                dx = dx.float()
        if wants_grad(weight):
            wgrad_accumulate(dy2, x2, weight)
            grad_ready(weight)
        if bias is not None and wants_grad(bias):
            bias_grad_accumulate(dy2, bias)
            grad_ready(bias)
        return dx, None, None


def _ceil8(n: int) -> int:
    return (n + 7) // 8 * 8


class _PaddedLinearFn(torch.autograd.Function):
    """Linear whose in/out features are not multiples of 8: the TMA-fed GEMMs
    need 16-byte row pitches, so operands are zero-padded to the next multiple
    of 8 (a copy of x, of the bf16 weight and of dy) and the results sliced."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        N, K = weight.shape
        Np, Kp = _ceil8(N), _ceil8(K)
        x2 = F.pad(as_bf16_2d(x), (0, Kp - K))
        w16 = F.pad(bf16_shadow(weight), (0, Kp - K, 0, Np - N))
        T = x2.shape[0]
        bias_p = F.pad(bias.detach().float(), (0, Np - N)) if bias is not None else None
        out = torch.empty((T, Np), device=x.device, dtype=torch.bfloat16)
        C().gemm(x2, w16, out, T, Np, Kp, False, False, bias=bias_p)
        ctx.save_for_backward(x2, w16, weight, bias)
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        return out[:, :N].reshape(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        x2, w16, weight, bias = ctx.saved_tensors
        N, K = weight.shape
        Np, Kp = w16.shape
        dyp = F.pad(as_bf16_2d(dy), (0, Np - N)).contiguous()
        T = dyp.shape[0]
        dx = None
        if ctx.needs_input_grad[0]:
            dx2 = torch.empty((T, Kp), device=dy.device, dtype=torch.bfloat16)
            C().gemm(dyp, w16, dx2, T, Kp, Np, False, True)
            dx = dx2[:, :K].to(ctx.x_dtype if ctx.x_dtype == torch.float32 else torch.bfloat16)
            dx = dx.reshape(ctx.x_shape)
        if wants_grad(weight):
            gp = torch.zeros((Np, Kp), device=dy.device, dtype=torch.float32)
            C().gemm(dyp, x2, gp, Np, Kp, T, True, True, flags=C().EPI_ACCUMULATE,
                     k_splits=splitk_for(Np, Kp, T))
            grad_buffer(weight).add_(gp[:N, :K])
            grad_ready(weight)
        if bias is not None and wants_grad(bias):
            C().colsum(dyp[:, :N], grad_buffer(bias))
            grad_ready(bias)
        return dx, None, None


_SMALL = {"tiles": None}


def set_small_gemm_tiles(n: Optional[int]) -> None:
    """Problems with fewer output tiles than ``n`` use the library GEMM
    (``None``: a quarter of the SMs; ``0``: always the tcgen05 kernels)."""
    _SMALL["tiles"] = n


def _few_tiles(M: int, N: int) -> bool:
    """Fewer 128x256 output tiles than the threshold (default: SMs / 4)."""
    if _SMALL["tiles"] is None:
        _SMALL["tiles"] = max(1, C().num_sms() // 4)
    return ((M + 127) // 128) * ((N + 255) // 256) < _SMALL["tiles"]


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           act: Optional[str] = None, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``act(x @ weight.T + bias) + residual``.

    CUDA inputs run the fused tcgen05 path (bf16 operands, f32 accumulation;
    the output is bf16, or f32 when a residual is added). CPU inputs run the
    plain PyTorch composition in the input dtype.
    """
    if not use_kernels(x):
        y = F.linear(x, weight, bias)
        if act == "gelu":
            y = F.gelu(y)
        elif act == "relu":
            y = F.relu(y)
        elif act is not None:
            raise ValueError(f"unsupported fused activation {act!r}")
        if residual is not None:
            y = residual + y
        return y
    if (weight.shape[0] % 8 == 0 and weight.shape[1] % 8 == 0
            and _few_tiles(x.numel() // x.shape[-1], weight.shape[0])):
        # A handful of output tiles would occupy a handful of SMs: the library
        # GEMM's split-K / small-tile kernels spread such problems over the
        # whole GPU. Same precision as the fused path (bf16 operands, f32
        # accumulation, bf16 output).
        y = _SmallLinearFn.apply(x, weight, bias)
        if act == "gelu":
            y = gelu_op(y)
        elif act == "relu":
            y = F.relu(y)
        elif act is not None:
            raise ValueError(f"unsupported fused activation {act!r}")
        return y if residual is None else residual + y
    if weight.shape[0] % 8 or weight.shape[1] % 8:
        y = _PaddedLinearFn.apply(x, weight, bias)
        if act == "gelu":
            y = gelu_op(y)
        elif act == "relu":
            y = F.relu(y)
        elif act is not None:
            raise ValueError(f"unsupported fused activation {act!r}")
        return y if residual is None else residual + y
    if act not in (None, "gelu"):
        y = _LinearFn.apply(x, weight, bias, None, None)
        y = F.relu(y) if act == "relu" else y
        return y if residual is None else residual + y
    return _LinearFn.apply(x, weight, bias, act, residual)
