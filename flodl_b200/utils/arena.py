"""Flat parameter arenas.

Parameters of a group are re-homed into one contiguous f32 buffer (and their
gradients into a second one), so a whole group is updated by ONE fused kernel
launch and a DDP bucket is a contiguous slice that a peer-memory collective can
address directly. Each parameter keeps its identity; only ``.data`` and
``.grad`` become views into the arena. A bf16 shadow arena mirrors the weights
for the forward GEMMs.

The allocator is pluggable: the peer-memory communicator passes an allocator
that returns symmetric (peer-mapped) buffers.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch

ALIGN = 64  # elements; keeps every view 256-byte aligned


def _round(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


class ParamArena:
    """Contiguous storage for a list of f32 parameters and their gradients."""

    def __init__(self, params: Sequence[torch.Tensor],
                 alloc: Optional[Callable[[int, torch.dtype, torch.device], torch.Tensor]] = None,
                 with_shadow: bool = True, grad_alloc=None):
        params = list(params)
        if not params:
            raise ValueError("ParamArena needs at least one parameter")
        dev = params[0].device
        for p in params:
            if p.dtype != torch.float32 or p.device != dev:
                raise ValueError("ParamArena parameters must be f32 on one device")
        self.params: List[torch.Tensor] = params
        self.device = dev
        self.offsets: List[int] = []
        off = 0
        for p in params:
            self.offsets.append(off)
            off += _round(p.numel())
        self.numel = off
        alloc = alloc or (lambda n, dt, d: torch.empty(n, dtype=dt, device=d))
        grad_alloc = grad_alloc or alloc
        self.data = alloc(self.numel, torch.float32, dev)
        self.grad = grad_alloc(self.numel, torch.float32, dev)
        with torch.no_grad():
            self.data.zero_()
            self.grad.zero_()
            for p, o in zip(params, self.offsets):
                n = p.numel()
                self.data[o:o + n].copy_(p.detach().reshape(-1))
                if p.grad is not None:
                    self.grad[o:o + n].copy_(p.grad.detach().reshape(-1))
        self.shadow = None
        if with_shadow and dev.type == "cuda":
            self.shadow = torch.empty(self.numel, dtype=torch.bfloat16, device=dev)
        self.rebind()
        self.refresh_shadow()
        for p in params:
            p._flodl_arena = self

    def view(self, buf: torch.Tensor, i: int) -> torch.Tensor:
        p = self.params[i]
        o = self.offsets[i]
        return buf[o:o + p.numel()].view(p.shape)

    def rebind(self) -> None:
        """Point every parameter's .data/.grad at the arena views."""
        from ..ops._common import set_shadow

        for i, p in enumerate(self.params):
            p.data = self.view(self.data, i)
            p.grad = self.view(self.grad, i)
            if self.shadow is not None:
                set_shadow(p, self.view(self.shadow, i))

    def is_bound(self) -> bool:
        for i, p in enumerate(self.params):
            if p.data_ptr() != self.data.data_ptr() + self.offsets[i] * 4:
                return False
            if p.grad is None or p.grad.data_ptr() != self.grad.data_ptr() + self.offsets[i] * 4:
                return False
        return True

    def refresh_shadow(self) -> None:
        if self.shadow is None:
            return
        from ..ops._common import C, mark_shadow_fresh

        with torch.no_grad():
            C().cast_f32_bf16(self.data, self.shadow)
        for p in self.params:
            mark_shadow_fresh(p)

    def zero_grad(self) -> None:
        with torch.no_grad():
            self.grad.zero_()
        for i, p in enumerate(self.params):
            if p.grad is None:
                p.grad = self.view(self.grad, i)

    def segment_of(self, p: torch.Tensor):
        for i, q in enumerate(self.params):
            if q is p:
                return self.offsets[i], p.numel()
        raise KeyError("parameter not in arena")


def arena_of(params: Sequence[torch.Tensor]) -> Optional[ParamArena]:
    """The arena that holds exactly ``params`` (in order), if any and still bound."""
    params = list(params)
    if not params:
        return None
    a = getattr(params[0], "_flodl_arena", None)
    if a is None or len(a.params) != len(params):
        return None
    if any(x is not y for x, y in zip(a.params, params)):
        return None
    return a if a.is_bound() else None
