"""Mixed precision helpers (flodl/src/nn/amp.rs).

The framework's fused CUDA ops already compute in bf16 with f32 accumulation
and f32 master weights; ``autocast`` is kept for modules that go through ATen
ops, and ``GradScaler`` for f16 training.
"""
from __future__ import annotations

import contextlib
import struct

import torch


@contextlib.contextmanager
def autocast(dtype: torch.dtype = torch.bfloat16, device_type: str = "cuda", enabled: bool = True):
    with torch.autocast(device_type=device_type, dtype=dtype, enabled=enabled):
        yield


class AutocastGuard:
    def __init__(self, dtype=torch.bfloat16, device_type="cuda"):
        self._cm = torch.autocast(device_type=device_type, dtype=dtype)
        self._cm.__enter__()

    def close(self):
        if self._cm is not None:
            self._cm.__exit__(None, None, None)
            self._cm = None

    def __del__(self):
        self.close()


def is_autocast_enabled(device_type: str = "cuda") -> bool:
    return torch.is_autocast_enabled(device_type)


is_autocast_enabled_for = is_autocast_enabled


def cast_parameters(module: torch.nn.Module, dtype: torch.dtype) -> None:
    with torch.no_grad():
        for p in module.parameters():
            p.data = p.data.to(dtype)


class GradScaler:
    """Dynamic loss scaling: scale the loss, unscale grads, skip steps with
    non-finite gradients, grow/back off the scale."""

    def __init__(self, init_scale: float = 2.0 ** 16, growth_factor: float = 2.0,
                 backoff_factor: float = 0.5, growth_interval: int = 2000):
        self.scale = init_scale
        self.growth_factor, self.backoff_factor = growth_factor, backoff_factor
        self.growth_interval = growth_interval
        self._growth_tracker = 0
        self._found_inf = False

    def scale_loss(self, loss):
        return loss * self.scale

    def unscale(self, optimizer) -> bool:
        inv = 1.0 / self.scale
        found = False
        for p in optimizer.params:
            if p.grad is not None:
                p.grad.mul_(inv)
                if not torch.isfinite(p.grad).all():
                    found = True
        self._found_inf = found
        return not found

    def step(self, optimizer) -> bool:
        ok = self.unscale(optimizer)
        if ok:
            optimizer.step()
        return ok

    def update(self) -> None:
        if self._found_inf:
            self.scale *= self.backoff_factor
            self._growth_tracker = 0
        else:
            self._growth_tracker += 1
            if self._growth_tracker >= self.growth_interval:
                self.scale *= self.growth_factor
                self._growth_tracker = 0

    def save_state(self, w):
        w.write(struct.pack("<dq", self.scale, self._growth_tracker))

    def load_state(self, r):
        self.scale, self._growth_tracker = struct.unpack("<dq", r.read(16))
