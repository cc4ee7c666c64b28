"""Fused softmax cross-entropy.

Reference: ``at::cross_entropy_loss`` with ``ignore_index`` and label smoothing
(flodl-sys/ops_training.cpp:1131, flodl/src/nn/loss.rs). The CUDA kernel
computes the mean loss and the logits gradient in the same pass; backward only
scales that gradient by the upstream scalar.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._common import C, use_kernels


class _SoftmaxCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, ignore_index, smoothing):
        l2 = logits.reshape(-1, logits.shape[-1])
        if l2.dtype != torch.bfloat16:
            l2 = l2.to(torch.bfloat16)
        l2 = l2.contiguous()
        t = targets.reshape(-1).to(torch.int64).contiguous()
        loss = torch.zeros((), device=logits.device, dtype=torch.float32)
        inv = torch.empty((), device=logits.device, dtype=torch.float32)
        dl = torch.empty_like(l2) if logits.requires_grad else None
        C().softmax_ce(l2, t, loss, inv, dl, int(ignore_index), float(smoothing))
        ctx.save_for_backward(dl)
        ctx.shape = logits.shape
        ctx.dtype = logits.dtype
        return loss

    @staticmethod
    def backward(ctx, g):
        (dl,) = ctx.saved_tensors
        grad = (dl * g.to(dl.dtype)).to(ctx.dtype).reshape(ctx.shape)
        return grad, None, None, None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100,
                  label_smoothing: float = 0.0) -> torch.Tensor:
    """Mean cross-entropy of ``logits [..., V]`` against integer ``targets``."""
    if not use_kernels(logits) or targets.dtype.is_floating_point:
        lg = logits.reshape(-1, logits.shape[-1])
        if lg.dtype in (torch.float16, torch.bfloat16):
            lg = lg.float()  # at least f32; f64 stays f64
        return F.cross_entropy(lg,
                               targets.reshape(-1) if not targets.dtype.is_floating_point
                               else targets.reshape(-1, targets.shape[-1]),
                               ignore_index=ignore_index, label_smoothing=label_smoothing)
    return _SoftmaxCEFn.apply(logits, targets, ignore_index, label_smoothing)


def softmax_ce_with_grad(logits_bf16: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100,
                         label_smoothing: float = 0.0):
    """Kernel entry used by fused model steps: returns (loss, dlogits of the mean loss)."""
    l2 = logits_bf16.reshape(-1, logits_bf16.shape[-1])
    t = targets.reshape(-1)
    loss = torch.zeros((), device=l2.device, dtype=torch.float32)
    inv = torch.empty((), device=l2.device, dtype=torch.float32)
    dl = torch.empty_like(l2)
    C().softmax_ce(l2, t, loss, inv, dl, int(ignore_index), float(label_smoothing))
    return loss, dl
