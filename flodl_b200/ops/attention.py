"""Scaled dot-product attention on packed QKV.

Reference: ``at::scaled_dot_product_attention`` (flodl-sys/ops_nn.cpp:407-431,
flodl/src/nn/attention.rs:136-230). The CUDA path runs the sm_100a flash
attention kernels (``_C.flash_attn_fwd`` / ``_C.flash_attn_bwd``): S = QK^T and
O += PV on tcgen05 with the accumulators in TMEM, online softmax, causal tile
skipping. Q/K/V are read straight out of the packed ``[T, 3C]`` projection
output and O is written as ``[T, C]`` (token-major), so no transposes run
around the kernel.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from ._common import C, use_kernels


def attn_fwd_packed(qkv: torch.Tensor, B: int, S: int, H: int, causal: bool,
                    key_padding: Optional[torch.Tensor] = None):
    """qkv [B*S, 3*H*D] bf16 -> (out [B*S, H*D] bf16, lse [B, H, S] f32)."""
    D = qkv.shape[1] // (3 * H)
    out = torch.empty((B * S, H * D), device=qkv.device, dtype=torch.bfloat16)
    lse = torch.empty((B, H, S), device=qkv.device, dtype=torch.float32)
    C().flash_attn_fwd(qkv, out, lse, B, S, H, D, bool(causal), 1.0 / math.sqrt(D), key_padding)
    return out, lse


def attn_bwd_packed(dout: torch.Tensor, qkv: torch.Tensor, out: torch.Tensor, lse: torch.Tensor,
                    B: int, S: int, H: int, causal: bool,
                    key_padding: Optional[torch.Tensor] = None,
                    bias_grad: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gradient of the packed QKV: dqkv [B*S, 3*H*D] bf16. With ``bias_grad``
    (f32 [3*H*D]) the column sums of dqkv - the gradient of the packed
    projection's bias - are accumulated into it in the same pass."""
    D = qkv.shape[1] // (3 * H)
    dqkv = torch.empty_like(qkv)
    C().flash_attn_bwd(dout.contiguous(), qkv, out, lse, dqkv, B, S, H, D, bool(causal),
                       1.0 / math.sqrt(D), key_padding, bias_grad)
    return dqkv


class _PackedAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, B, S, H, causal, key_padding):
        out, lse = attn_fwd_packed(qkv, B, S, H, causal, key_padding)
        ctx.save_for_backward(qkv, out, lse, key_padding)
        ctx.dims = (B, S, H, causal)
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, out, lse, key_padding = ctx.saved_tensors
        B, S, H, causal = ctx.dims
        d16 = dout if dout.dtype == torch.bfloat16 else dout.to(torch.bfloat16)
        return attn_bwd_packed(d16, qkv, out, lse, B, S, H, causal, key_padding), None, None, None, None, None


def attention_packed(qkv: torch.Tensor, B: int, S: int, H: int, causal: bool = False,
                     key_padding: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Self-attention over packed ``qkv [B*S, 3C]``; returns ``[B*S, C]``.

    ``key_padding`` (bool ``[B, S]``, True = masked key) implements the padding
    mask used by BERT-style encoders.
    """
    if not use_kernels(qkv):
        D = qkv.shape[1] // (3 * H)
        q, k, v = qkv.view(B, S, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
        mask = None
        if key_padding is not None:
            mask = ~key_padding[:, None, None, :]
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=causal and mask is None)
        return o.permute(0, 2, 1, 3).reshape(B * S, H * D)
    q16 = qkv if qkv.dtype == torch.bfloat16 else qkv.to(torch.bfloat16)
    return _PackedAttnFn.apply(q16.contiguous(), B, S, H, causal, key_padding)


def scaled_dot_product_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                 attn_mask: Optional[torch.Tensor] = None, is_causal: bool = False,
                                 dropout_p: float = 0.0) -> torch.Tensor:
    """Functional SDPA on ``[B, H, S, D]`` tensors (floDl's functional API).

    Self-attention with head size 64 (the flash kernel's) runs the kernel
    through the packed layout when there is no mask or the mask only hides
    keys (boolean, broadcast over heads and queries: ``[B, 1, 1, S]`` with
    True = attend, the padding mask of encoder batches); anything else uses
    the composed (explicit softmax) form, which is also the CPU path.
    """
    B, H, S, D = q.shape
    key_padding = None
    if (attn_mask is not None and attn_mask.dtype == torch.bool and attn_mask.dim() == 4
            and attn_mask.shape[1] == 1 and attn_mask.shape[2] == 1
            and attn_mask.shape[0] in (1, B) and attn_mask.shape[3] == S and not is_causal):
        key_padding = (~attn_mask[:, 0, 0, :]).expand(B, S).contiguous()
    if (q.is_cuda and (attn_mask is None or key_padding is not None) and dropout_p == 0.0
            and k.shape == q.shape and v.shape == q.shape and D == 64):
        qkv = torch.stack([q, k, v], dim=0).permute(1, 3, 0, 2, 4).reshape(B * S, 3 * H * D)
        o = attention_packed(qkv.to(torch.bfloat16), B, S, H, is_causal, key_padding)
        return o.view(B, S, H, D).permute(0, 2, 1, 3).to(q.dtype)
    scale = 1.0 / math.sqrt(D)
    s = torch.matmul(q, k.transpose(-2, -1)) * scale
    if is_causal:
        m = torch.ones(S, k.shape[-2], dtype=torch.bool, device=q.device).tril()
        s = s.masked_fill(~m, float("-inf"))
    if attn_mask is not None:
        if attn_mask.dtype == torch.bool:
            s = s.masked_fill(~attn_mask, float("-inf"))
        else:
            s = s + attn_mask
    p = torch.softmax(s.float(), dim=-1).to(q.dtype)
    if dropout_p > 0:
        p = F.dropout(p, dropout_p)
    return torch.matmul(p, v)
