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


def _pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


def _pack_weight(weight, cin_pad):
    """OIHW f32 -> bf16 [Cout, kh*kw*cin_pad], column (kh*kw_ + kw)*cin_pad + ci."""
    w = weight.detach().permute(0, 2, 3, 1)
    if cin_pad != w.shape[-1]:
        w = F.pad(w, (0, cin_pad - w.shape[-1]))
    return w.reshape(w.shape[0], -1).to(torch.bfloat16).contiguous()


def _to_nhwc(x, cin_pad):
    xh = x.permute(0, 2, 3, 1)
    if cin_pad != xh.shape[-1]:
        xh = F.pad(xh, (0, cin_pad - xh.shape[-1]))
    return xh.to(torch.bfloat16).contiguous()


class _Conv2dFn(torch.autograd.Function):
    """Square-kernel 2-D convolution (groups 1, dilation 1) on the tcgen05 GEMM:
    im2col (columns (kh, kw, ci)) -> GEMM with the packed weight; backward =
    dgrad GEMM + col2im and a split-K weight-gradient GEMM. NCHW in/out (the
    output is a channels-last NCHW view, bf16)."""

    @staticmethod
    def forward(ctx, x, weight, bias, stride, padding):
        K_ = C()
        N, Cin, H, W = x.shape
        Cout, _, k, _ = weight.shape
        cp = (Cin + 7) // 8 * 8
        s, p = stride, padding
        Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
        M, Kc = N * Ho * Wo, k * k * cp
        xh = _to_nhwc(x, cp)
        if k == 1 and s == 1 and p == 0:
            cols = xh.view(M, Kc)
        else:
            cols = torch.empty((M, Kc), device=x.device, dtype=torch.bfloat16)
            K_.im2col(xh, cols, k, s, p)
        wp = _pack_weight(weight, cp)
        y = torch.empty((M, Cout), device=x.device, dtype=torch.bfloat16)
        K_.gemm(cols, wp, y, M, Cout, Kc, False, False,
                bias=bias.detach().float().contiguous() if bias is not None else None)
        ctx.save_for_backward(cols, wp, weight, bias)
        ctx.geo = (N, Cin, cp, H, W, Ho, Wo, k, s, p, x.dtype)
        return y.view(N, Ho, Wo, Cout).permute(0, 3, 1, 2)

    @staticmethod
    def backward(ctx, dy):
        K_ = C()
        cols, wp, weight, bias = ctx.saved_tensors
        N, Cin, cp, H, W, Ho, Wo, k, s, p, xdt = ctx.geo
        Cout = weight.shape[0]
        M, Kc = N * Ho * Wo, k * k * cp
        dyh = dy.permute(0, 2, 3, 1).to(torch.bfloat16).contiguous().view(M, Cout)
        dx = None
        if ctx.needs_input_grad[0]:
            dcols = torch.empty((M, Kc), device=dy.device, dtype=torch.bfloat16)
            K_.gemm(dyh, wp, dcols, M, Kc, Cout, False, True)
            dxh = torch.empty((N, H, W, cp), device=dy.device, dtype=torch.bfloat16)
            K_.col2im(dcols, dxh, k, s, p)
            dx = dxh[..., :Cin].permute(0, 3, 1, 2).to(xdt)
        if wants_grad(weight):
            gp = torch.zeros((Cout, Kc), device=dy.device, dtype=torch.float32)
            K_.gemm(dyh, cols, gp, Cout, Kc, M, True, True, flags=K_.EPI_ACCUMULATE,
                    k_splits=_splitk(Cout, Kc, M))
            g = gp.view(Cout, k, k, cp)[..., :Cin].permute(0, 3, 1, 2)
            grad_buffer(weight).add_(g)
            grad_ready(weight)
        if bias is not None and wants_grad(bias):
            K_.colsum(dyh, grad_buffer(bias))
            grad_ready(bias)
        return dx, None, None, None, None


def _splitk(m, n, k):
    from ._common import splitk_for
    return splitk_for(m, n, k)


def conv2d(x, weight, bias=None, stride=1, padding=0, dilation=1, groups=1):
    """2-D convolution. CUDA inputs with square kernels, equal strides and
    paddings, groups 1, dilation 1 and a multiple of 8 output channels run
    the tcgen05 path; everything else PyTorch's convolution."""
    st, pd, dl = _pair(stride), _pair(padding), _pair(dilation)
    k = weight.shape[-1]
    fast = (use_kernels(x) and x.dim() == 4 and groups == 1 and dl == (1, 1)
            and weight.shape[-2] == k and st[0] == st[1] and pd[0] == pd[1]
            and weight.shape[0] % 8 == 0 and isinstance(pd[0], int))
    if not fast:
        return F.conv2d(x, weight, bias, stride, padding, dilation, groups)
    return _Conv2dFn.apply(x, weight, bias, st[0], pd[0])


class _BatchNorm2dFn(torch.autograd.Function):
    """Training-mode batch norm over an NCHW tensor with the NHWC kernels
    (statistics + running update, apply; backward reduce + apply)."""

    @staticmethod
    def forward(ctx, x, weight, bias, running_mean, running_var, momentum, eps):
        K_ = C()
        N, Cc, H, W = x.shape
        xh = x.permute(0, 2, 3, 1).to(torch.bfloat16).contiguous().view(-1, Cc)
        ws = torch.zeros(2 * Cc + 1, device=x.device, dtype=torch.float32)
        mean = torch.empty(Cc, device=x.device)
        rstd = torch.empty(Cc, device=x.device)
        K_.bn_stats(xh, mean, rstd, running_mean, running_var, ws, eps, momentum)
        y = torch.empty_like(xh)
        K_.bn_apply(xh, mean, rstd, weight.detach() if weight is not None else None,
                    bias.detach() if bias is not None else None, None, False, y)
        ctx.save_for_backward(xh, mean, rstd, weight, bias, ws)
        ctx.shape, ctx.dtype = (N, Cc, H, W), x.dtype
        return y.view(N, H, W, Cc).permute(0, 3, 1, 2)

    @staticmethod
    def backward(ctx, dy):
        K_ = C()
        xh, mean, rstd, weight, bias, ws = ctx.saved_tensors
        N, Cc, H, W = ctx.shape
        dyh = dy.permute(0, 2, 3, 1).to(torch.bfloat16).contiguous().view(-1, Cc)
        dx = torch.empty_like(xh)
        sums = torch.empty(2 * Cc, device=dy.device)
        dg = grad_buffer(weight) if weight is not None and wants_grad(weight) else None
        db = grad_buffer(bias) if bias is not None and wants_grad(bias) else None
        K_.bn_bwd(dyh, None, xh, mean, rstd, weight.detach() if weight is not None else None,
                  dg, db, sums, ws, dx)
        if dg is not None:
            grad_ready(weight)
        if db is not None:
            grad_ready(bias)
        return dx.view(N, H, W, Cc).permute(0, 3, 1, 2).to(ctx.dtype), None, None, None, None, None, None


def batch_norm2d(x, running_mean, running_var, weight, bias, training, momentum, eps):
    """BatchNorm2d. CUDA tensors in training mode with a multiple of 8
    channels run the NHWC sm_100a kernels; otherwise PyTorch's batch norm."""
    if (use_kernels(x) and training and x.dim() == 4 and x.shape[1] % 8 == 0
            and x.shape[1] <= 2048):
        return _BatchNorm2dFn.apply(x, weight, bias, running_mean, running_var, momentum, eps)
    return F.batch_norm(x, running_mean, running_var, weight, bias, training, momentum, eps)
