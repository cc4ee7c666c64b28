"""Layers (reference: flodl/src/nn/*.rs).

Linear, LayerNorm, MultiheadAttention and Embedding run the sm_100a kernels on
CUDA; the rest are thin modules over ATen ops with floDl's constructors,
defaults and ``name()`` identifiers.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple, Union

import torch
import torch.nn.functional as F

from .. import ops
from . import init as _init
from .module import Module, NamedInputModule

_Int2 = Union[int, Tuple[int, int]]


def _pair(v) -> Tuple[int, int]:
    return (v, v) if isinstance(v, int) else tuple(v)


def _dev(device):
    return torch.device(device) if device is not None else torch.device("cpu")


class Identity(Module):
    NAME = "identity"

    def forward(self, x):
        return x


# ---------------------------------------------------------------- Linear
class Linear(Module):
    """``y = x W^T + b`` (flodl/src/nn/linear.rs). Init: kaiming-uniform(a=sqrt 5),
    bias uniform(+-1/sqrt(in)). CUDA forward is one tcgen05 GEMM."""

    NAME = "linear"

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        dev = _dev(device)
        self.weight = torch.nn.Parameter(
            _init.kaiming_uniform((out_features, in_features), in_features, math.sqrt(5.0), dev))
        self.bias = (torch.nn.Parameter(_init.uniform_bias(in_features, (out_features,), dev))
                     if bias else None)

    @classmethod
    def no_bias(cls, in_features: int, out_features: int, device=None) -> "Linear":
        return cls(in_features, out_features, bias=False, device=device)

    def forward(self, x):
        return ops.linear(x, self.weight, self.bias)


class Bilinear(Module):
    NAME = "bilinear"

    def __init__(self, in1: int, in2: int, out: int, bias: bool = True, device=None):
        super().__init__()
        bound = 1.0 / math.sqrt(in1)
        dev = _dev(device)
        self.weight = torch.nn.Parameter(torch.empty(out, in1, in2, device=dev).uniform_(-bound, bound))
        self.bias = torch.nn.Parameter(torch.empty(out, device=dev).uniform_(-bound, bound)) if bias else None

    def forward(self, x1, x2=None):
        if x2 is None:
            x1, x2 = x1
        return F.bilinear(x1, x2, self.weight, self.bias)


# ---------------------------------------------------------------- conv
class _ConvNd(Module):
    def __init__(self, nd, in_ch, out_ch, kernel_size, stride=1, padding=0, dilation=1, groups=1,
                 bias=True, transposed=False, output_padding=0, device=None):
        super().__init__()
        tup = (lambda v: (v,) * nd if isinstance(v, int) else tuple(v))
        self.nd = nd
        self.kernel_size = tup(kernel_size)
        self.stride = tup(stride)
        self.padding = tup(padding)
        self.dilation = tup(dilation)
        self.output_padding = tup(output_padding)
        self.groups = groups
        self.transposed = transposed
        dev = _dev(device)
        if transposed:
            wshape = (in_ch, out_ch // groups) + self.kernel_size
            fan_in = (out_ch // groups) * math.prod(self.kernel_size)
        else:
            wshape = (out_ch, in_ch // groups) + self.kernel_size
            fan_in = (in_ch // groups) * math.prod(self.kernel_size)
        self.weight = torch.nn.Parameter(_init.kaiming_uniform(wshape, fan_in, math.sqrt(5.0), dev))
        self.bias = torch.nn.Parameter(_init.uniform_bias(fan_in, (out_ch,), dev)) if bias else None

    def _lib_operands(self, x):
        """Library-path convolutions follow the activation's precision: a bf16
        activation (from a tcgen05 layer) meets a bf16 cast of the f32 master
        weight, as under autocast; f32 activations use the weight as is."""
        w, b = self.weight, self.bias
        if x.dtype != w.dtype and x.dtype in (torch.bfloat16, torch.float16):
            w = w.to(x.dtype)
            b = b.to(x.dtype) if b is not None else None
        elif x.dtype != w.dtype:
            x = x.to(w.dtype)
        return x, w, b

    def forward(self, x):
        if self.transposed:
            if self.nd in (1, 2) and x.is_cuda:
                fn = ops.conv_transpose2d if self.nd == 2 else ops.conv_transpose1d
                return fn(x, self.weight, self.bias, self.stride, self.padding,
                          self.output_padding, self.groups, self.dilation)
            fn = {1: F.conv_transpose1d, 2: F.conv_transpose2d, 3: F.conv_transpose3d}[self.nd]
            x, w, b = self._lib_operands(x)
            return fn(x, w, b, self.stride, self.padding, self.output_padding, self.groups,
                      self.dilation)
        if self.nd == 2:
            return ops.conv2d(x, self.weight, self.bias, self.stride, self.padding, self.dilation,
                              self.groups)
        if self.nd == 1 and x.is_cuda:
            return ops.conv1d(x, self.weight, self.bias, self.stride, self.padding,
                              self.dilation, self.groups)
        fn = {1: F.conv1d, 3: F.conv3d}[self.nd]
        x, w, b = self._lib_operands(x)
        return fn(x, w, b, self.stride, self.padding, self.dilation, self.groups)


class Conv1d(_ConvNd):
    NAME = "conv1d"

    def __init__(self, in_ch, out_ch, kernel_size, stride=1, padding=0, dilation=1, groups=1,
                 bias=True, device=None):
        super().__init__(1, in_ch, out_ch, kernel_size, stride, padding, dilation, groups, bias,
                         device=device)


class Conv2d(_ConvNd):
    """2-D convolution (flodl/src/nn/conv2d.rs). 3x3 NHWC bf16 convolutions run
    the implicit-GEMM tcgen05 kernel on CUDA."""

    NAME = "conv2d"

    def __init__(self, in_ch, out_ch, kernel_size, stride=1, padding=0, dilation=1, groups=1,
                 bias=True, device=None):
        super().__init__(2, in_ch, out_ch, kernel_size, stride, padding, dilation, groups, bias,
                         device=device)


class Conv3d(_ConvNd):
    NAME = "conv3d"

    def __init__(self, in_ch, out_ch, kernel_size, stride=1, padding=0, dilation=1, groups=1,
                 bias=True, device=None):
        super().__init__(3, in_ch, out_ch, kernel_size, stride, padding, dilation, groups, bias,
                         device=device)


class ConvTranspose1d(_ConvNd):
    NAME = "conv_transpose1d"

    def __init__(self, in_ch, out_ch, kernel_size, stride=1, padding=0, output_padding=0,
                 dilation=1, groups=1, bias=True, device=None):
        super().__init__(1, in_ch, out_ch, kernel_size, stride, padding, dilation, groups, bias,
                         True, output_padding, device=device)


class ConvTranspose2d(_ConvNd):
    NAME = "conv_transpose2d"

    def __init__(self, in_ch, out_ch, kernel_size, stride=1, padding=0, output_padding=0,
                 dilation=1, groups=1, bias=True, device=None):
        super().__init__(2, in_ch, out_ch, kernel_size, stride, padding, dilation, groups, bias,
                         True, output_padding, device=device)


class ConvTranspose3d(_ConvNd):
    NAME = "conv_transpose3d"

    def __init__(self, in_ch, out_ch, kernel_size, stride=1, padding=0, output_padding=0,
                 dilation=1, groups=1, bias=True, device=None):
        super().__init__(3, in_ch, out_ch, kernel_size, stride, padding, dilation, groups, bias,
                         True, output_padding, device=device)


# ---------------------------------------------------------------- pooling & reshaping
class MaxPool2d(Module):
    NAME = "maxpool2d"

    def __init__(self, kernel_size, stride=None, padding=0, dilation=1, ceil_mode=False):
        super().__init__()
        self.args = (kernel_size, stride if stride is not None else kernel_size, padding, dilation,
                     ceil_mode)

    def forward(self, x):
        from ..ops import max_pool2d
        k, s, p, d, c = self.args
        return max_pool2d(x, k, s, p, d, c)


class MaxPool1d(MaxPool2d):
    NAME = "maxpool1d"

    def forward(self, x):
        from ..ops import max_pool1d
        k, s, p, d, c = self.args
        return max_pool1d(x, k, s, p, d, c)


class AvgPool2d(Module):
    NAME = "avgpool2d"

    def __init__(self, kernel_size, stride=None, padding=0, ceil_mode=False, count_include_pad=True):
        super().__init__()
        self.args = (kernel_size, stride if stride is not None else kernel_size, padding, ceil_mode,
                     count_include_pad)

    def forward(self, x):
        return F.avg_pool2d(x, *self.args)


class AvgPool1d(AvgPool2d):
    NAME = "avgpool1d"

    def forward(self, x):
        return F.avg_pool1d(x, *self.args)


class AdaptiveAvgPool2d(Module):
    NAME = "adaptive_avgpool2d"

    def __init__(self, output_size):
        super().__init__()
        self.output_size = output_size

    def forward(self, x):
        return F.adaptive_avg_pool2d(x, self.output_size)


class AdaptiveMaxPool2d(AdaptiveAvgPool2d):
    NAME = "adaptive_maxpool2d"

    def forward(self, x):
        return F.adaptive_max_pool2d(x, self.output_size)


class PixelShuffle(Module):
    NAME = "pixel_shuffle"

    def __init__(self, upscale_factor: int):
        super().__init__()
        self.r = upscale_factor

    def forward(self, x):
        return F.pixel_shuffle(x, self.r)


class PixelUnshuffle(PixelShuffle):
    NAME = "pixel_unshuffle"

    def forward(self, x):
        return F.pixel_unshuffle(x, self.r)


class Upsample(Module):
    NAME = "upsample"

    def __init__(self, size=None, scale_factor=None, mode: str = "nearest", align_corners=None):
        super().__init__()
        self.size, self.scale_factor, self.mode, self.align_corners = size, scale_factor, mode, align_corners

    def forward(self, x):
        return F.interpolate(x, self.size, self.scale_factor, self.mode, self.align_corners)


class Unfold(Module):
    NAME = "unfold"

    def __init__(self, kernel_size, dilation=1, padding=0, stride=1):
        super().__init__()
        self.args = (kernel_size, dilation, padding, stride)

    def forward(self, x):
        return F.unfold(x, *self.args)


class Fold(Module):
    NAME = "fold"

    def __init__(self, output_size, kernel_size, dilation=1, padding=0, stride=1):
        super().__init__()
        self.args = (output_size, kernel_size, dilation, padding, stride)

    def forward(self, x):
        return F.fold(x, *self.args)


class Flatten(Module):
    NAME = "flatten"

    def __init__(self, start_dim: int = 1, end_dim: int = -1):
        super().__init__()
        self.start_dim, self.end_dim = start_dim, end_dim

    def forward(self, x):
        return torch.flatten(x, self.start_dim, self.end_dim)


class ZeroPad2d(Module):
    NAME = "zeropad2d"

    def __init__(self, padding):
        super().__init__()
        self.padding = (padding,) * 4 if isinstance(padding, int) else tuple(padding)

    def forward(self, x):
        return F.pad(x, self.padding, mode="constant", value=0.0)


class ReflectionPad2d(ZeroPad2d):
    NAME = "reflectionpad2d"

    def forward(self, x):
        return F.pad(x, self.padding, mode="reflect")


class GaussianBlur(Module):
    """Separable Gaussian blur over [N, C, H, W] (flodl/src/nn/functional.rs)."""

    NAME = "gaussian_blur"

    def __init__(self, kernel_size: int, sigma: float):
        super().__init__()
        self.kernel_size, self.sigma = kernel_size, sigma

    def forward(self, x):
        return gaussian_blur_2d(x, self.kernel_size, self.sigma)


def gaussian_blur_2d(x: torch.Tensor, kernel_size: int, sigma: float) -> torch.Tensor:
    half = kernel_size // 2
    t = torch.arange(kernel_size, dtype=x.dtype, device=x.device) - half
    k = torch.exp(-0.5 * (t / sigma) ** 2)
    k = k / k.sum()
    C = x.shape[1]
    kh = k.view(1, 1, kernel_size, 1).repeat(C, 1, 1, 1)
    kw = k.view(1, 1, 1, kernel_size).repeat(C, 1, 1, 1)
    x = F.conv2d(F.pad(x, (0, 0, half, half), mode="reflect"), kh, groups=C)
    return F.conv2d(F.pad(x, (half, half, 0, 0), mode="reflect"), kw, groups=C)


# ---------------------------------------------------------------- normalisation
class LayerNorm(Module):
    """LayerNorm over the last dim (flodl/src/nn/layernorm.rs), eps 1e-5 default.
    CUDA runs the fused one-pass kernel."""

    NAME = "layernorm"
    DEFAULT_EPS = 1e-5

    def __init__(self, size: int, eps: float = DEFAULT_EPS, device=None):
        super().__init__()
        dev = _dev(device)
        self.size = size
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.ones(size, device=dev))
        self.bias = torch.nn.Parameter(torch.zeros(size, device=dev))

    @classmethod
    def with_eps(cls, size: int, eps: float, device=None) -> "LayerNorm":
        return cls(size, eps, device)

    def forward(self, x):
        return ops.layer_norm(x, self.weight, self.bias, self.eps)


class RMSNorm(Module):
    NAME = "rmsnorm"

    def __init__(self, size: int, eps: float = 1e-5, device=None):
        super().__init__()
        self.eps = eps  # the reference's default (flodl/src/nn/rmsnorm.rs:39)
        self.weight = torch.nn.Parameter(torch.ones(size, device=_dev(device)))

    def forward(self, x):
        from ..ops import rms_norm
        return rms_norm(x, self.weight, self.eps)


class GroupNorm(Module):
    NAME = "groupnorm"

    def __init__(self, num_groups: int, num_channels: int, eps: float = 1e-5, affine: bool = True,
                 device=None):
        super().__init__()
        self.num_groups, self.eps = num_groups, eps
        dev = _dev(device)
        self.weight = torch.nn.Parameter(torch.ones(num_channels, device=dev)) if affine else None
        self.bias = torch.nn.Parameter(torch.zeros(num_channels, device=dev)) if affine else None

    def forward(self, x):
        from ..ops import group_norm
        return group_norm(x, self.num_groups, self.weight, self.bias, self.eps)


class BatchNorm(Module):
    """BatchNorm over [N, C] or [N, C, L] (flodl/src/nn/batchnorm.rs). Running
    statistics are f32 buffers (they ride the cluster-averaging collective)."""

    NAME = "batchnorm"

    def __init__(self, num_features: int, eps: float = 1e-5, momentum: float = 0.1,
                 affine: bool = True, device=None):
        super().__init__()
        dev = _dev(device)
        self.num_features, self.eps, self.momentum = num_features, eps, momentum
        self.weight = torch.nn.Parameter(torch.ones(num_features, device=dev)) if affine else None
        self.bias = torch.nn.Parameter(torch.zeros(num_features, device=dev)) if affine else None
        self.register_buffer("running_mean", torch.zeros(num_features, device=dev))
        self.register_buffer("running_var", torch.ones(num_features, device=dev))

    def forward(self, x):
        return F.batch_norm(x, self.running_mean, self.running_var, self.weight, self.bias,
                            self.training, self.momentum, self.eps)


class BatchNorm2d(BatchNorm):
    NAME = "batchnorm2d"

    def forward(self, x):
        return ops.batch_norm2d(x, self.running_mean, self.running_var, self.weight, self.bias,
                                self.training, self.momentum, self.eps)


class InstanceNorm(Module):
    NAME = "instancenorm"

    def __init__(self, num_features: int, eps: float = 1e-5, affine: bool = False, device=None):
        super().__init__()
        dev = _dev(device)
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.ones(num_features, device=dev)) if affine else None
        self.bias = torch.nn.Parameter(torch.zeros(num_features, device=dev)) if affine else None

    def forward(self, x):
        return F.instance_norm(x, weight=self.weight, bias=self.bias, eps=self.eps)


# ---------------------------------------------------------------- dropout
class Dropout(Module):
    NAME = "dropout"

    def __init__(self, p: float = 0.5):
        super().__init__()
        self.p = p

    def forward(self, x):
        from ..ops import dropout
        return dropout(x, self.p, self.training)


class Dropout2d(Dropout):
    NAME = "dropout2d"

    def forward(self, x):
        return F.dropout2d(x, self.p, self.training)


class AlphaDropout(Dropout):
    NAME = "alpha_dropout"

    def forward(self, x):
        return F.alpha_dropout(x, self.p, self.training)


# ---------------------------------------------------------------- embedding
class Embedding(Module):
    """Lookup table (flodl/src/nn/embedding.rs), N(0,1) init, optional padding_idx."""

    NAME = "embedding"

    def __init__(self, num_embeddings: int, embedding_dim: int, padding_idx: Optional[int] = None,
                 device=None):
        super().__init__()
        w = torch.randn(num_embeddings, embedding_dim, device=_dev(device))
        if padding_idx is not None:
            w[padding_idx].zero_()
        self.padding_idx = padding_idx
        self.weight = torch.nn.Parameter(w)

    def forward(self, ids):
        return ops.embedding(ids, self.weight, self.padding_idx)


class EmbeddingBag(Module):
    NAME = "embedding_bag"

    def __init__(self, num_embeddings: int, embedding_dim: int, mode: str = "mean", device=None):
        super().__init__()
        self.mode = mode
        self.weight = torch.nn.Parameter(torch.randn(num_embeddings, embedding_dim, device=_dev(device)))

    def forward(self, ids, offsets=None):
        return F.embedding_bag(ids, self.weight, offsets, mode=self.mode)


# ---------------------------------------------------------------- recurrent
class _RNNBase(Module):
    def __init__(self, cls, input_size, hidden_size, num_layers=1, batch_first=True, device=None):
        super().__init__()
        self.rnn = cls(input_size, hidden_size, num_layers=num_layers, batch_first=batch_first,
                       device=_dev(device))
        self.state = None

    def forward(self, x, state=None):
        out, st = self.rnn(x, state if state is not None else self.state)
        self.state = st
        return out

    def reset(self):
        self.state = None

    def detach_state(self):
        if self.state is None:
            return
        if isinstance(self.state, tuple):
            self.state = tuple(s.detach() for s in self.state)
        else:
            self.state = self.state.detach()


class GRU(_RNNBase):
    """Multi-layer GRU over cuDNN's fused kernel (flodl/src/nn/gru.rs)."""

    NAME = "gru"

    def __init__(self, input_size, hidden_size, num_layers=1, batch_first=True, device=None):
        super().__init__(torch.nn.GRU, input_size, hidden_size, num_layers, batch_first, device)


class LSTM(_RNNBase):
    NAME = "lstm"

    def __init__(self, input_size, hidden_size, num_layers=1, batch_first=True, device=None):
        super().__init__(torch.nn.LSTM, input_size, hidden_size, num_layers, batch_first, device)


class GRUCell(Module):
    NAME = "grucell"

    def __init__(self, input_size, hidden_size, device=None):
        super().__init__()
        self.cell = torch.nn.GRUCell(input_size, hidden_size, device=_dev(device))
        self.h = None

    def forward(self, x, h=None):
        self.h = self.cell(x, h if h is not None else self.h)
        return self.h

    def reset(self):
        self.h = None

    def detach_state(self):
        if self.h is not None:
            self.h = self.h.detach()


class LSTMCell(Module):
    NAME = "lstmcell"

    def __init__(self, input_size, hidden_size, device=None):
        super().__init__()
        self.cell = torch.nn.LSTMCell(input_size, hidden_size, device=_dev(device))
        self.state = None

    def forward(self, x, state=None):
        h, c = self.cell(x, state if state is not None else self.state)
        self.state = (h, c)
        return h

    def reset(self):
        self.state = None

    def detach_state(self):
        if self.state is not None:
            self.state = tuple(s.detach() for s in self.state)


# ---------------------------------------------------------------- attention
class MultiheadAttention(NamedInputModule):
    """Multi-head attention (flodl/src/nn/attention.rs:28,136-230).

    Self-attention packs Q/K/V into one projection GEMM and runs the sm_100a
    flash kernel on the packed buffer. Cross-attention (``using`` a tagged
    memory) projects K/V from the memory tensor.
    """

    NAME = "multihead_attention"

    def __init__(self, embed_dim: int, num_heads: int, causal: bool = False, device=None):
        super().__init__()
        assert embed_dim % num_heads == 0
        self.embed_dim, self.num_heads, self.causal = embed_dim, num_heads, causal
        dev = _dev(device)
        self.qkv = Linear(embed_dim, 3 * embed_dim, device=dev)
        self.out_proj = Linear(embed_dim, embed_dim, device=dev)

    def forward_named(self, x, refs):
        memory = None
        if refs:
            memory = next(iter(refs.values()))
        return self.attend(x, memory)

    def forward(self, x, refs=None, key_padding_mask=None):
        if isinstance(refs, torch.Tensor):
            return self.attend(x, refs, key_padding_mask)
        return self.attend(x, next(iter(refs.values())) if refs else None, key_padding_mask)

    def attend(self, x, memory=None, key_padding_mask=None):
        B, S, Cd = x.shape
        H = self.num_heads
        D = Cd // H
        if memory is None:
            qkv = self.qkv(x.reshape(B * S, Cd))
            o = ops.attention_packed(qkv, B, S, H, self.causal, key_padding_mask)
        else:
            Wq, Wk, Wv = self.qkv.weight.chunk(3, 0)
            bq, bk, bv = (self.qkv.bias.chunk(3, 0) if self.qkv.bias is not None else (None,) * 3)
            q = ops.linear(x, Wq, bq).view(B, S, H, D).transpose(1, 2)
            Sm = memory.shape[1]
            k = ops.linear(memory, Wk, bk).view(B, Sm, H, D).transpose(1, 2)
            v = ops.linear(memory, Wv, bv).view(B, Sm, H, D).transpose(1, 2)
            mask = None if key_padding_mask is None else ~key_padding_mask[:, None, None, :]
            o = ops.scaled_dot_product_attention(q, k, v, mask, self.causal and S == Sm)
            o = o.transpose(1, 2).reshape(B * S, Cd)
        return self.out_proj(o).reshape(B, S, Cd).to(x.dtype)


class RotaryEmbedding(Module):
    """Rotary position embedding applied to [B, H, S, D] (flodl/src/nn/rope.rs)."""

    NAME = "rope"

    def __init__(self, dim: int, max_seq: int = 4096, base: float = 10000.0, device=None):
        super().__init__()
        inv = 1.0 / (base ** (torch.arange(0, dim, 2, device=_dev(device)).float() / dim))
        t = torch.arange(max_seq, device=_dev(device)).float()
        freqs = torch.outer(t, inv)
        self.register_buffer("cos", freqs.cos(), persistent=False)
        self.register_buffer("sin", freqs.sin(), persistent=False)

    def forward(self, x, offset: int = 0):
        S = x.shape[-2]
        cos = self.cos[offset:offset + S].to(x.dtype)
        sin = self.sin[offset:offset + S].to(x.dtype)
        x1, x2 = x[..., 0::2], x[..., 1::2]
        out = torch.stack((x1 * cos - x2 * sin, x1 * sin + x2 * cos), dim=-1)
        return out.flatten(-2)
