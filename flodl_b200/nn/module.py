"""Module system.

Mirrors floDl's ``Module`` trait (flodl/src/nn/mod.rs:139-330) on top of
``torch.nn.Module`` so tensors, autograd and device moves come from PyTorch:

* ``name()``            lowercase identifier used as graph node-id prefix
* ``parameters()``      learnable parameters, deduplicated by identity
* ``buffers()``         persistent non-learnable state
* ``sub_modules()``     direct children
* ``move_to_device()``  move params/buffers, keeping parameter identity
* ``set_training()``    train/eval
* ``trace()``, ``reset()``, ``detach_state()``  loop/recurrent hooks
* ``structural_hash()`` only composite graphs return one

floDl names a parameter by its short local name (``weight``, ``bias``);
``named_parameters`` of a :class:`~flodl_b200.graph.Graph` prefixes it with the
node's tag or id ("encoder/weight"). ``Parameter`` and ``Buffer`` are plain
``torch`` tensors here; their local name is the attribute name.
"""
from __future__ import annotations

from typing import Iterator, List, Optional, Tuple

import torch


class Module(torch.nn.Module):
    """Base class of every layer and composite in the framework."""

    #: lowercase identifier used to derive graph node ids (``linear_1``)
    NAME = "module"

    def name(self) -> str:
        return self.NAME

    # --------------------------------------------------------------- params
    def parameters(self, recurse: bool = True) -> List[torch.nn.Parameter]:  # type: ignore[override]
        seen = set()
        out = []
        for p in super().parameters(recurse=recurse):
            if id(p) not in seen:
                seen.add(id(p))
                out.append(p)
        return out

    def buffers(self, recurse: bool = True) -> List[torch.Tensor]:  # type: ignore[override]
        seen = set()
        out = []
        for b in super().buffers(recurse=recurse):
            if id(b) not in seen:
                seen.add(id(b))
                out.append(b)
        return out

    def local_named_parameters(self) -> List[Tuple[str, torch.nn.Parameter]]:
        """(local name, parameter) pairs, e.g. ``[("weight", W), ("bias", b)]``.

        Nested children's parameters are named ``child.weight``.
        """
        return list(super().named_parameters())

    def local_named_buffers(self) -> List[Tuple[str, torch.Tensor]]:
        return list(super().named_buffers())

    def sub_modules(self) -> List["Module"]:
        return [m for m in self.children()]

    # --------------------------------------------------------------- device
    def move_to_device(self, device) -> "Module":
        """Move parameters and buffers in place (parameter identity is kept)."""
        device = torch.device(device)
        with torch.no_grad():
            for p in self.parameters():
                if p.device != device:
                    p.data = p.data.to(device)
                    if p.grad is not None:
                        p.grad = p.grad.to(device)
            for mod in self.modules():
                for k, b in list(mod._buffers.items()):
                    if b is not None and b.device != device:
                        mod._buffers[k] = b.to(device)
        return self

    def device(self) -> torch.device:
        for p in self.parameters():
            return p.device
        for b in self.buffers():
            return b.device
        return torch.device("cpu")

    # --------------------------------------------------------------- mode
    def set_training(self, training: bool) -> None:
        self.train(training)

    def is_training(self) -> bool:
        return self.training

    # --------------------------------------------------------------- hooks
    def trace(self) -> Optional[torch.Tensor]:
        return None

    def reset(self) -> None:
        for m in self.sub_modules():
            if isinstance(m, Module):
                m.reset()

    def detach_state(self) -> None:
        for m in self.sub_modules():
            if isinstance(m, Module):
                m.detach_state()

    def structural_hash(self) -> Optional[str]:
        return None

    def as_named_input(self):
        """Return self if this module accepts named extra inputs (``using``)."""
        return None

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())


class NamedInputModule(Module):
    """A module that receives extra tagged inputs via ``FlowBuilder.using``.

    ``forward_named(x, refs)`` gets the main stream and a dict tag -> tensor
    (reference: ``NamedInputModule``, flodl/src/nn/mod.rs:389).
    """

    def forward_named(self, x, refs):  # pragma: no cover - interface
        raise NotImplementedError

    def as_named_input(self):
        return self

    def forward(self, x, refs=None):
        return self.forward_named(x, refs or {})


def walk_modules(m: torch.nn.Module) -> Iterator[torch.nn.Module]:
    """Depth-first walk over a module tree, each module once."""
    seen = set()
    stack = [m]
    while stack:
        cur = stack.pop()
        if id(cur) in seen:
            continue
        seen.add(id(cur))
        yield cur
        stack.extend(reversed(list(cur.children())))
