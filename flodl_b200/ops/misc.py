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
    """2-D convolution (groups 1, dilation 1, any kh x kw kernel with per-axis
    stride and padding) on the tcgen05 GEMM: im2col (columns (kh, kw, ci)) ->
    GEMM with the packed weight; backward = dgrad GEMM + col2im and a split-K
    weight-gradient GEMM. NCHW in/out (the output is a channels-last NCHW
    view, bf16). 1-D convolutions run as kh = 1 (flodl-sys/ops_nn.cpp:19-275
    routes every convolution through one entry the same way)."""

    @staticmethod
    def forward(ctx, x, weight, bias, stride, padding):
        K_ = C()
        N, Cin, H, W = x.shape
        # a 1-D weight [Cout, Cin, k] is the 1 x k kernel; the gradient goes
        # to the weight as given (the parameter itself, not a view of it)
        Cout, kh, kw = weight.shape[0], (weight.shape[2] if weight.dim() == 4 else 1), weight.shape[-1]
        cp = (Cin + 7) // 8 * 8
        (sh, sw), (ph, pw) = stride, padding
        Ho, Wo = (H + 2 * ph - kh) // sh + 1, (W + 2 * pw - kw) // sw + 1
        M, Kc = N * Ho * Wo, kh * kw * cp
        xh = _to_nhwc(x, cp)
        if kh == 1 and kw == 1 and sh == 1 and sw == 1 and ph == 0 and pw == 0:
            cols = xh.view(M, Kc)
        else:
            cols = torch.empty((M, Kc), device=x.device, dtype=torch.bfloat16)
            K_.im2col_geo(xh, cols, kh, kw, sh, sw, ph, pw)
        wp = _pack_weight(weight.view(Cout, -1, kh, kw), cp)
        y = torch.empty((M, Cout), device=x.device, dtype=torch.bfloat16)
        K_.gemm(cols, wp, y, M, Cout, Kc, False, False,
                bias=bias.detach().float().contiguous() if bias is not None else None)
        ctx.save_for_backward(cols, wp, weight, bias)
        ctx.geo = (N, Cin, cp, H, W, Ho, Wo, kh, kw, sh, sw, ph, pw, x.dtype)
        return y.view(N, Ho, Wo, Cout).permute(0, 3, 1, 2)

    @staticmethod
    def backward(ctx, dy):
        K_ = C()
        cols, wp, weight, bias = ctx.saved_tensors
        N, Cin, cp, H, W, Ho, Wo, kh, kw, sh, sw, ph, pw, xdt = ctx.geo
        Cout = weight.shape[0]
        M, Kc = N * Ho * Wo, kh * kw * cp
        dyh = dy.permute(0, 2, 3, 1).to(torch.bfloat16).contiguous().view(M, Cout)
        dx = None
        if ctx.needs_input_grad[0]:
            dcols = torch.empty((M, Kc), device=dy.device, dtype=torch.bfloat16)
            K_.gemm(dyh, wp, dcols, M, Kc, Cout, False, True)
            dxh = torch.empty((N, H, W, cp), device=dy.device, dtype=torch.bfloat16)
            K_.col2im_geo(dcols, dxh, kh, kw, sh, sw, ph, pw)
            dx = dxh[..., :Cin].permute(0, 3, 1, 2).to(xdt)
        if wants_grad(weight):
            gp = torch.zeros((Cout, Kc), device=dy.device, dtype=torch.float32)
            K_.gemm(dyh, cols, gp, Cout, Kc, M, True, True, flags=K_.EPI_ACCUMULATE,
                    k_splits=_splitk(Cout, Kc, M))
            g = gp.view(Cout, kh, kw, cp)[..., :Cin].permute(0, 3, 1, 2)
            grad_buffer(weight).add_(g.reshape(weight.shape))
            grad_ready(weight)
        if bias is not None and wants_grad(bias):
            K_.colsum(dyh, grad_buffer(bias))
            grad_ready(bias)
        return dx, None, None, None, None


def _splitk(m, n, k):
    from ._common import splitk_for
    return splitk_for(m, n, k)


def conv2d(x, weight, bias=None, stride=1, padding=0, dilation=1, groups=1):
    """2-D convolution. CUDA inputs with groups 1, dilation 1, integer
    paddings and a multiple of 8 output channels run the tcgen05 path (any
    kh x kw kernel, per-axis stride and padding); everything else PyTorch's
    convolution."""
    st, pd, dl = _pair(stride), _pair(padding), _pair(dilation)
    fast = (use_kernels(x) and x.dim() == 4 and groups == 1 and dl == (1, 1)
            and weight.shape[0] % 8 == 0 and all(isinstance(v, int) for v in pd))
    if not fast:
        return F.conv2d(x, weight, bias, stride, padding, dilation, groups)
    return _Conv2dFn.apply(x, weight, bias, st, pd)


def conv1d(x, weight, bias=None, stride=1, padding=0, dilation=1, groups=1):
    """1-D convolution over [N, C, L] as a 1 x k 2-D convolution on the
    tcgen05 path (same conditions as :func:`conv2d`)."""
    s = stride if isinstance(stride, int) else stride[0]
    p = padding if isinstance(padding, int) else padding[0]
    d = dilation if isinstance(dilation, int) else dilation[0]
    if not (use_kernels(x) and x.dim() == 3 and groups == 1 and d == 1 and isinstance(p, int)
            and weight.shape[0] % 8 == 0):
        return F.conv1d(x, weight, bias, stride, padding, dilation, groups)
    y = _Conv2dFn.apply(x.unsqueeze(2), weight, bias, (1, s), (0, p))
    return y.squeeze(2)


class _ConvTranspose2dFn(torch.autograd.Function):
    """Transposed 2-D convolution (groups 1, dilation 1) on the tcgen05 GEMM.
    Its forward is a convolution's data gradient: with the weight [Cin, Cout,
    kh, kw] read as the weight of a convolution from Cout to Cin channels,
    cols = x (NHWC rows) x packed weight, then col2im onto the output grid.
    Backward: the input gradient is that convolution's forward (im2col of dy,
    GEMM), the weight gradient a split-K GEMM of x against those columns."""

    @staticmethod
    def forward(ctx, x, weight, bias, stride, padding, output_padding):
        K_ = C()
        N, Cin, H, W = x.shape
        # a 1-D weight [Cin, Cout, k] is the 1 x k kernel (gradient to the weight as given)
        w4 = weight if weight.dim() == 4 else weight.unsqueeze(2)
        Cout, kh, kw = w4.shape[1], w4.shape[2], w4.shape[3]
        (sh, sw), (ph, pw), (oh, ow) = stride, padding, output_padding
        Hout = (H - 1) * sh - 2 * ph + kh + oh
        Wout = (W - 1) * sw - 2 * pw + kw + ow
        cp = (Cout + 7) // 8 * 8
        M, Kc = N * H * W, kh * kw * cp
        xh = x.permute(0, 2, 3, 1).to(torch.bfloat16).contiguous().view(M, Cin)
        wp = _pack_weight(w4, cp)  # [Cin, kh*kw*cp]: the convolution Cout -> Cin
        cols = torch.empty((M, Kc), device=x.device, dtype=torch.bfloat16)
        K_.gemm(xh, wp, cols, M, Kc, Cin, False, True)
        yh = torch.empty((N, Hout, Wout, cp), device=x.device, dtype=torch.bfloat16)
        K_.col2im_geo(cols, yh, kh, kw, sh, sw, ph, pw)
        y = yh[..., :Cout]
        if bias is not None:
            y = (y.float() + bias.detach().float()).to(torch.bfloat16)
        ctx.save_for_backward(xh, wp, weight, bias)
        ctx.geo = (N, Cin, Cout, cp, H, W, Hout, Wout, kh, kw, sh, sw, ph, pw, x.dtype)
        return y.permute(0, 3, 1, 2)

    @staticmethod
    def backward(ctx, dy):
        K_ = C()
        xh, wp, weight, bias = ctx.saved_tensors
        N, Cin, Cout, cp, H, W, Hout, Wout, kh, kw, sh, sw, ph, pw, xdt = ctx.geo
        M, Kc = N * H * W, kh * kw * cp
        dyh = _to_nhwc(dy, cp)  # [N, Hout, Wout, cp]
        cols = torch.empty((M, Kc), device=dy.device, dtype=torch.bfloat16)
        K_.im2col_geo(dyh, cols, kh, kw, sh, sw, ph, pw)
        dx = None
        if ctx.needs_input_grad[0]:
            dxh = torch.empty((M, Cin), device=dy.device, dtype=torch.bfloat16)
            K_.gemm(cols, wp, dxh, M, Cin, Kc, False, False)
            dx = dxh.view(N, H, W, Cin).permute(0, 3, 1, 2).to(xdt)
        if wants_grad(weight):
            gp = torch.zeros((Cin, Kc), device=dy.device, dtype=torch.float32)
            K_.gemm(xh, cols, gp, Cin, Kc, M, True, True, flags=K_.EPI_ACCUMULATE,
                    k_splits=_splitk(Cin, Kc, M))
            g = gp.view(Cin, kh, kw, cp)[..., :Cout].permute(0, 3, 1, 2)
            grad_buffer(weight).add_(g.reshape(weight.shape))
            grad_ready(weight)
        if bias is not None and wants_grad(bias):
            K_.colsum(dyh.view(-1, cp)[:, :Cout], grad_buffer(bias))
            grad_ready(bias)
        return dx, None, None, None, None, None


def conv_transpose2d(x, weight, bias=None, stride=1, padding=0, output_padding=0, groups=1,
                     dilation=1):
    """Transposed 2-D convolution; CUDA inputs with groups 1, dilation 1 and a
    multiple of 8 input channels run the tcgen05 path, everything else
    PyTorch's."""
    st, pd, op, dl = _pair(stride), _pair(padding), _pair(output_padding), _pair(dilation)
    fast = (use_kernels(x) and x.dim() == 4 and groups == 1 and dl == (1, 1)
            and weight.shape[0] % 8 == 0 and all(isinstance(v, int) for v in pd + op)
            and op[0] < st[0] and op[1] < st[1])
    if not fast:
        return F.conv_transpose2d(x, weight, bias, stride, padding, output_padding, groups,
                                  dilation)
    return _ConvTranspose2dFn.apply(x, weight, bias, st, pd, op)


def conv_transpose1d(x, weight, bias=None, stride=1, padding=0, output_padding=0, groups=1,
                     dilation=1):
    """Transposed 1-D convolution as a 1 x k transposed 2-D convolution."""
    one = lambda v: v if isinstance(v, int) else v[0]
    s, p, o, d = one(stride), one(padding), one(output_padding), one(dilation)
    if not (use_kernels(x) and x.dim() == 3 and groups == 1 and d == 1 and isinstance(p, int)
            and weight.shape[0] % 8 == 0 and o < s):
        return F.conv_transpose1d(x, weight, bias, stride, padding, output_padding, groups,
                                  dilation)
    y = _ConvTranspose2dFn.apply(x.unsqueeze(2), weight, bias, (1, s), (0, p), (0, o))
    return y.squeeze(2)


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


def _pool_out(n, k, s, p, d, ceil_mode):
    span = n + 2 * p - d * (k - 1) - 1
    o = (-(-span // s) if ceil_mode else span // s) + 1
    if ceil_mode and (o - 1) * s >= n + p:  # the last window must start inside the input
        o -= 1
    return o


class _MaxPool2dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, k, s, p, d, ceil_mode):
        xc = x.contiguous()
        H, W = xc.shape[-2:]
        Ho = _pool_out(H, k[0], s[0], p[0], d[0], ceil_mode)
        Wo = _pool_out(W, k[1], s[1], p[1], d[1], ceil_mode)
        y = torch.empty(xc.shape[:-2] + (Ho, Wo), device=x.device, dtype=x.dtype)
        idx = torch.empty(y.shape, device=x.device, dtype=torch.int32)
        C().maxpool_fwd(xc, y, idx, k[0], k[1], s[0], s[1], p[0], p[1], d[0], d[1])
        ctx.save_for_backward(idx)
        ctx.in_shape = xc.shape
        return y

    @staticmethod
    def backward(ctx, dy):
        (idx,) = ctx.saved_tensors
        dx = torch.zeros(ctx.in_shape, device=dy.device, dtype=dy.dtype)
        C().maxpool_bwd(dy.contiguous(), idx, dx)
        return dx, None, None, None, None, None


def max_pool2d(x, kernel_size, stride=None, padding=0, dilation=1, ceil_mode=False):
    """Max pooling over the last two dimensions (flodl/src/nn/pooling.rs): one
    kernel forward (with the argmax of each window), one scatter backward, for
    f32 and bf16 on CUDA; PyTorch's elsewhere."""
    k = _pair(kernel_size)
    s = _pair(stride if stride is not None else kernel_size)
    p, d = _pair(padding), _pair(dilation)
    if not use_kernels(x) or x.dtype not in (torch.float32, torch.bfloat16) or x.dim() < 3:
        return F.max_pool2d(x, k, s, p, d, ceil_mode)
    return _MaxPool2dFn.apply(x, k, s, p, d, bool(ceil_mode))


def max_pool1d(x, kernel_size, stride=None, padding=0, dilation=1, ceil_mode=False):
    """Max pooling over the last dimension through the 2-D kernel (H = 1)."""
    if not use_kernels(x) or x.dtype not in (torch.float32, torch.bfloat16) or x.dim() < 2:
        return F.max_pool1d(x, kernel_size, stride, padding, dilation, ceil_mode)
    st = stride if stride is not None else kernel_size
    y = max_pool2d(x.unsqueeze(-2), (1, kernel_size), (1, st), (0, padding), (1, dilation),
                   ceil_mode)
    return y.squeeze(-2)


_DROPOUT_CALLS = [0]


class _DropoutFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, p, seed, offset):
        xc = x.contiguous()
        y = torch.empty_like(xc)
        C().dropout(xc, y, p, seed, offset)
        ctx.args = (p, seed, offset)
        return y

    @staticmethod
    def backward(ctx, dy):
        p, seed, offset = ctx.args
        dyc = dy.contiguous()
        dx = torch.empty_like(dyc)
        C().dropout(dyc, dx, p, seed, offset)  # the same mask and scale
        return dx, None, None, None


def dropout(x: torch.Tensor, p: float = 0.5, training: bool = True) -> torch.Tensor:
    """Dropout (flodl/src/nn/dropout.rs). On CUDA (f32/bf16, outside CUDA-graph
    capture) one kernel draws the mask from a counter-based generator keyed by
    a seed from torch's generator, so the backward regenerates it instead of
    keeping it; under capture, and elsewhere, PyTorch's (which advances its
    generator per graph replay)."""
    if not training or p == 0.0:
        return x
    if (not use_kernels(x) or x.dtype not in (torch.float32, torch.bfloat16) or p >= 1.0
            or torch.cuda.is_current_stream_capturing()):
        return F.dropout(x, p, training)
    seed = int(torch.randint(0, 2 ** 62, (1,)).item())
    _DROPOUT_CALLS[0] += 1
    return _DropoutFn.apply(x, float(p), seed, _DROPOUT_CALLS[0])
