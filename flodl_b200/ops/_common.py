"""Shared plumbing of the fused op layer.

* ``use_kernels(t)``: the sm_100a kernels run for CUDA tensors; CPU tensors take
  the plain PyTorch path (the CPU device path of the framework, and the fp32
  numerics oracle for the kernel tests).
* bf16 weight shadows: forward GEMMs read a bf16 copy of each f32 master weight.
  The fused optimizers refresh the shadow in the same pass as the update, so the
  cast never runs as a separate kernel in steady state. A shadow is rebuilt when
  the parameter's version counter moved (a torch in-place op touched it).
* side-effect gradient accumulation: the backward of a fused op accumulates the
  f32 weight gradient straight into ``param.grad`` (split-K tcgen05 GEMM with
  ``red.global.add``) and then notifies the gradient-ready listeners (the DDP
  bucket reducer) for that parameter. The autograd graph sees ``None`` for such
  weights, which is how the fused collective overlaps with backward.
"""
from __future__ import annotations

from typing import Callable, List

import torch

from .._ext import cuda_ext



def use_kernels(t: torch.Tensor) -> bool:
    return t.is_cuda


def C():
    return cuda_ext()


# ----------------------------------------------------------------- shadows
def bf16_shadow(p: torch.Tensor) -> torch.Tensor:
    """bf16 copy of an f32 CUDA parameter, cached on the parameter object."""
    if p.dtype == torch.bfloat16:
        return p.detach()
    sh = getattr(p, "_flodl_bf16", None)
    ver = p._version
    if sh is None or sh.shape != p.shape or sh.device != p.device:
        sh = torch.empty(p.shape, dtype=torch.bfloat16, device=p.device)
        p._flodl_bf16 = sh
        p._flodl_bf16_ver = -1
    if getattr(p, "_flodl_bf16_ver", -1) != ver or getattr(p, "_flodl_bf16_ptr", 0) != p.data_ptr():
        with torch.no_grad():
            src = p.detach()
            if not src.is_contiguous():
                src = src.contiguous()
            C().cast_f32_bf16(src, sh)
        p._flodl_bf16_ver = ver
        p._flodl_bf16_ptr = p.data_ptr()
    return sh


def set_shadow(p: torch.Tensor, shadow: torch.Tensor) -> None:
    """Adopt an externally maintained bf16 shadow (e.g. a slice of a flat arena)."""
    p._flodl_bf16 = shadow
    p._flodl_bf16_ver = p._version
    p._flodl_bf16_ptr = p.data_ptr()


def mark_shadow_fresh(p: torch.Tensor) -> None:
    """Declare the shadow current after a kernel rewrote both copies in place."""
    if getattr(p, "_flodl_bf16", None) is not None:
        p._flodl_bf16_ver = p._version
        p._flodl_bf16_ptr = p.data_ptr()


# ----------------------------------------------------------------- grads
def grad_buffer(p: torch.Tensor) -> torch.Tensor:
    """The f32 gradient buffer of ``p``, created zeroed on first use."""
    if p.grad is None:
        p.grad = torch.zeros_like(p, dtype=torch.float32, memory_format=torch.contiguous_format)
    return p.grad


def add_grad_ready_listener(p: torch.Tensor, fn: Callable[[torch.Tensor], None]) -> None:
    # stored on the parameter itself (tensors cannot be dict keys: == is elementwise)
    ls = getattr(p, "_flodl_grad_listeners", None)
    if ls is None:
        ls = []
        p._flodl_grad_listeners = ls
    ls.append(fn)


def clear_grad_ready_listeners(p: torch.Tensor) -> None:
    p._flodl_grad_listeners = []


def grad_ready(p: torch.Tensor) -> None:
    """Called after a fused backward finished accumulating ``p.grad``."""
    for fn in getattr(p, "_flodl_grad_listeners", ()):
        fn(p)


def wants_grad(p) -> bool:
    return p is not None and isinstance(p, torch.Tensor) and p.requires_grad


def splitk_for(m: int, n: int, k: int) -> int:
    """Split-K factor for a weight-gradient GEMM with a long reduction."""
    tiles = ((m + 127) // 128) * ((n + 255) // 256)
    sms = C().num_sms()
    if tiles >= sms:
        return 1
    ks = max(1, min(sms // max(tiles, 1), k // 512))
    return ks


def as_bf16_2d(t: torch.Tensor) -> torch.Tensor:
    t2 = t.reshape(-1, t.shape[-1])
    if t2.dtype != torch.bfloat16:
        out = torch.empty(t2.shape, dtype=torch.bfloat16, device=t2.device)
        C().cast_f32_bf16(t2.float().contiguous(), out)
        return out
    return t2.contiguous()
