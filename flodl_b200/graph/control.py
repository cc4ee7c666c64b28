"""Loops, routing (gate/switch), map, routers and halting conditions.

References: flodl/src/graph/loop_node.rs, gate.rs, switch.rs, map.rs,
router.rs, halt.rs.

* loops: ``for_n(n)``, ``while_cond(cond, max)`` (checks before each
  iteration), ``until_cond(cond, max)`` (checks after); the condition module
  returns a scalar, > 0 means "halt" for until and "continue" for while. Each
  iteration's body output (or ``trace()``) is recorded as a loop trace.
* gate: all experts run; the router's ``[..., E]`` weights combine them
  (stack, broadcast, sum).
* switch: the router picks a branch (scalar index for the batch, or one index
  per row); only selected branches run.
* map: apply the body to each element along dim 0 (``each``), to a tagged
  tensor (``over``), or to ``n`` slices; ``batched()`` runs the body once on
  the whole batch when it is element-wise.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from ..nn.layers import Linear
from ..nn.module import Module


def _scalar(t: torch.Tensor, it: int) -> float:
    if t.numel() != 1:
        raise ValueError(f"loop condition at iteration {it}: condition returned {t.numel()} values "
                         f"(shape {list(t.shape)}) but the loop halts for the whole batch — reduce "
                         "the condition to a single scalar")
    return float(t.detach().reshape(()).item())


class LoopComposite(Module):
    NAME = "loop"

    def __init__(self, body: torch.nn.Module, mode: str, n: int, cond: Optional[torch.nn.Module] = None):
        super().__init__()
        self.body = body
        self.cond = cond
        self.mode = mode
        self.n = n
        self.traces: List[torch.Tensor] = []
        self.iterations = 0

    def _trace(self, out):
        t = self.body.trace() if hasattr(self.body, "trace") else None
        self.traces.append(t if t is not None else out)

    def forward(self, x):
        if hasattr(self.body, "reset"):
            self.body.reset()
        self.traces = []
        it = 0
        if self.mode == "for":
            for it in range(self.n):
                x = self.body(x)
                self._trace(x)
            self.iterations = self.n
            return x
        if self.mode == "while":
            while it < self.n and _scalar(self.cond(x), it) > 0.0:
                x = self.body(x)
                self._trace(x)
                it += 1
            self.iterations = it
            return x
        # until
        while it < self.n:
            x = self.body(x)
            self._trace(x)
            it += 1
            if _scalar(self.cond(x), it) > 0.0:
                break
        self.iterations = it
        return x


class LoopBuilder:
    def __init__(self, fb, body):
        self.fb = fb
        self.body = body

    def _wire(self, comp: LoopComposite):
        fb = self.fb
        if not fb._single("loop"):
            return fb
        prev = fb.current[0]
        from .flow import Node

        ref = fb._add_node(Node(fb.next_id("loop"), "loop", comp))
        fb._edge(prev, ref.node_id)
        fb.current = [ref]
        fb.on_target = ref
        return fb

    def for_n(self, n: int):
        if n < 1:
            self.fb.fail("loop requires at least 1 iteration")
            return self.fb
        return self._wire(LoopComposite(self.body, "for", n))

    def while_cond(self, cond, max_iter: int):
        if max_iter < 1:
            self.fb.fail("loop requires max_iter >= 1")
            return self.fb
        return self._wire(LoopComposite(self.body, "while", max_iter, cond))

    def until_cond(self, cond, max_iter: int):
        if max_iter < 1:
            self.fb.fail("loop requires max_iter >= 1")
            return self.fb
        return self._wire(LoopComposite(self.body, "until", max_iter, cond))


class GateComposite(Module):
    NAME = "gate"

    def __init__(self, router, experts: Sequence[torch.nn.Module]):
        super().__init__()
        self.router = router
        self.experts = torch.nn.ModuleList(experts)

    def forward(self, x):
        w = self.router(x)  # [..., E]
        outs = torch.stack([e(x) for e in self.experts], dim=-1)  # [..., D, E]
        while w.dim() < outs.dim():
            w = w.unsqueeze(-2)
        return (outs * w).sum(-1)


class SwitchComposite(Module):
    NAME = "switch"

    def __init__(self, router, branches: Sequence[torch.nn.Module]):
        super().__init__()
        self.router = router
        self.branches = torch.nn.ModuleList(branches)

    def forward(self, x):
        sel = self.router(x)
        if sel.numel() == 1:
            i = int(sel.reshape(()).item())
            if not 0 <= i < len(self.branches):
                raise IndexError(f"switch: router selected branch {i} of {len(self.branches)}")
            return self.branches[i](x)
        idx = sel.reshape(-1).long()
        out = None
        for b in torch.unique(idx).tolist():
            rows = (idx == b).nonzero(as_tuple=True)[0]
            y = self.branches[b](x.index_select(0, rows))
            if out is None:
                out = y.new_zeros((x.shape[0],) + tuple(y.shape[1:]))
            out = out.index_copy(0, rows, y)
        return out


class MapComposite(Module):
    NAME = "map"

    def __init__(self, body, batched: bool, slices: int = 0):
        super().__init__()
        self.body = body
        self.batched = batched
        self.slices = slices

    def forward(self, x):
        if self.slices:
            parts = torch.chunk(x, self.slices, dim=-1)
            if self.batched:
                return torch.cat(self.body(torch.stack(parts, 0)).unbind(0), dim=-1)
            return torch.cat([self.body(p) for p in parts], dim=-1)
        if self.batched:
            return self.body(x)
        return torch.stack([self.body(e) for e in x.unbind(0)], 0)


class MapBuilder:
    def __init__(self, fb, body):
        self.fb = fb
        self.body = body
        self._batched = False

    def batched(self):
        self._batched = True
        return self

    def each(self):
        return self.fb._composite("map", MapComposite(self.body, self._batched))

    def over(self, tag: str):
        src = self.fb.taps.get(tag)
        if src is None:
            self.fb.fail(f"Map.over({tag!r}) references unknown tag; Map requires a backward reference")
            return self.fb
        return self.fb._composite("map", MapComposite(self.body, self._batched), source=src)

    def slices(self, n: int):
        if n < 1:
            self.fb.fail(f"Map.slices requires n >= 1 (got {n})")
            return self.fb
        return self.fb._composite("map", MapComposite(self.body, self._batched, n))


# ---------------------------------------------------------------- routers
def _wide(t: torch.Tensor) -> torch.Tensor:
    """At least f32 for the routing math (bf16/f16 widen; f32/f64 stay)."""
    return t.float() if t.dtype in (torch.float16, torch.bfloat16) else t


class SoftmaxRouter(Module):
    NAME = "softmax_router"

    def __init__(self, input_dim: int, num_experts: int, device=None):
        super().__init__()
        self.proj = Linear(input_dim, num_experts, device=device)

    def forward(self, x):
        return torch.softmax(_wide(self.proj(x)), dim=-1).to(x.dtype)


class SigmoidRouter(SoftmaxRouter):
    NAME = "sigmoid_router"

    def forward(self, x):
        return torch.sigmoid(_wide(self.proj(x))).to(x.dtype)


class FixedSelector(Module):
    NAME = "fixed_selector"

    def __init__(self, index: int):
        super().__init__()
        self.index = index

    def forward(self, x):
        return torch.tensor(float(self.index), device=x.device)


class ArgmaxSelector(Module):
    NAME = "argmax_selector"

    def __init__(self, input_dim: int, num_branches: int, device=None):
        super().__init__()
        self.proj = Linear(input_dim, num_branches, device=device)

    def forward(self, x):
        return self.proj(x).argmax(dim=-1)


# ---------------------------------------------------------------- halting
class ThresholdHalt(Module):
    """Halt when the mean of the stream exceeds ``threshold`` (returns > 0)."""

    NAME = "threshold_halt"

    def __init__(self, threshold: float):
        super().__init__()
        self.threshold = threshold

    def forward(self, x):
        return x.float().mean() - self.threshold


class LearnedHalt(Module):
    """Learned halting score: mean sigmoid(Wx) - 0.5."""

    NAME = "learned_halt"

    def __init__(self, input_dim: int, device=None):
        super().__init__()
        self.proj = Linear(input_dim, 1, device=device)

    def forward(self, x):
        return torch.sigmoid(_wide(self.proj(x))).mean() - 0.5
