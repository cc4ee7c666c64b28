"""Tensor/device helpers. Tensors and autograd are libtorch's (as in floDl:
flodl/src/tensor/mod.rs, flodl/src/autograd/). ``Variable`` is a tensor that
may require grad; ``no_grad`` / ``NoGradGuard`` disable graph recording."""
from __future__ import annotations

import contextlib

import torch

Tensor = torch.Tensor
Variable = torch.Tensor
DType = torch.dtype


class Device:
    CPU = torch.device("cpu")

    @staticmethod
    def cuda(i: int = 0) -> torch.device:
        return torch.device("cuda", i)


def test_device() -> torch.device:
    """CUDA(0) when a GPU is present, else CPU (flodl/src/tensor/mod.rs:1511)."""
    return torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")


def manual_seed(seed: int) -> None:
    torch.manual_seed(seed)


no_grad = torch.no_grad


class NoGradGuard:
    def __init__(self):
        self._cm = torch.no_grad()
        self._cm.__enter__()

    def close(self):
        if self._cm is not None:
            self._cm.__exit__(None, None, None)
            self._cm = None

    def __del__(self):
        self.close()


def gpu_memory_stats(device=0) -> dict:
    if not torch.cuda.is_available():
        return {}
    free, total = torch.cuda.mem_get_info(device)
    return {"free": free, "total": total, "allocated": torch.cuda.memory_allocated(device),
            "reserved": torch.cuda.memory_reserved(device)}
