"""Host-fed training step runner (public API).

``StepRunner`` owns static device input buffers and a training-step callable,
optionally captured once as a CUDA graph. ``step(*host_tensors)`` copies the
step's inputs from (pinned) host memory into the static buffers on the
current stream, runs the step (graph replay or eager), and returns the loss
read back to the host. This is the end-to-end path a user runs; the device
copy/replay/readback are the only per-step work besides the kernels.
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch


class StepRunner:
    def __init__(self, step_fn: Callable[[], torch.Tensor], inputs: Sequence[torch.Tensor],
                 graph: Optional[torch.cuda.CUDAGraph] = None,
                 graph_loss: Optional[torch.Tensor] = None):
        self.step_fn = step_fn
        self.inputs = list(inputs)
        self.graph = graph
        self.graph_loss = graph_loss

    @classmethod
    def for_state(cls, state, graph_step=None, eager_step=None) -> "StepRunner":
        g, l = graph_step if graph_step is not None else (None, None)
        inputs = state["inputs"] if "inputs" in state else [state["ids"], state["tgt"]]
        return cls(eager_step, inputs, g, l)

    @classmethod
    def capture(cls, step_fn: Callable[[], torch.Tensor], inputs: Sequence[torch.Tensor],
                warmup: int = 3) -> "StepRunner":
        """Warm up ``step_fn`` then capture it as a CUDA graph."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                step_fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        # captured on the warm-up stream: autograd nodes that outlive a warm-up
        # step (loop traces, cached gradient accumulators) record the stream
        # they were created on, and a captured backward that syncs with a
        # stream outside the capture is invalid
        with torch.cuda.graph(g, stream=s):
            loss = step_fn()
        return cls(step_fn, inputs, g, loss)

    @classmethod
    def capture_training(cls, model, optimizer, loss_fn, example_inputs: Sequence[torch.Tensor],
                         warmup: int = 3) -> "StepRunner":
        """Capture ``loss_fn(model(x), y)`` + backward + ``optimizer.step()`` +
        ``zero_grad`` as one CUDA graph over static input buffers (copies of
        ``example_inputs``). The warm-up steps (on a side stream) create the
        optimizer's flat arena and device scalars, so the captured step
        allocates nothing and syncs with the host nowhere. Models whose
        forward makes host-side decisions (``while``/``until`` loops, hard
        switches) cannot be captured; the capture then raises."""
        static = [t.detach().clone() for t in example_inputs]

        def step():
            out = model(*static[:-1])
            loss = loss_fn(out, static[-1])
            loss.backward()
            optimizer.step()
            optimizer.zero_grad()
            return loss.detach()

        return cls.capture(step, static, warmup)

    def replay(self, *device_inputs: torch.Tensor) -> torch.Tensor:
        """Device-side step: copy inputs into the static buffers, replay,
        return the loss tensor (no host sync)."""
        for dst, src in zip(self.inputs, device_inputs):
            dst.copy_(src, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            return self.graph_loss
        return self.step_fn()

    def step(self, *host_inputs: torch.Tensor) -> float:
        if len(host_inputs) != len(self.inputs):
            raise ValueError(f"expected {len(self.inputs)} inputs, got {len(host_inputs)}")
        for dst, src in zip(self.inputs, host_inputs):
            dst.copy_(src, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            loss = self.graph_loss
        else:
            loss = self.step_fn()
        return float(loss.item())

    def step_pipelined(self, *host_inputs: torch.Tensor) -> Optional[float]:
        """One step whose loss is read back one step late: the inputs are
        copied in (pinned host memory -> device, asynchronous), the step is
        launched, its loss is copied into a pinned host slot behind an event,
        and the PREVIOUS step's loss is returned (None on the first call) once
        its event completed. The host never waits for the step it just
        launched, so the next step's copies and launch overlap this step's
        execution; every step's loss still reaches the host. ``flush()``
        returns the last one."""
        if len(host_inputs) != len(self.inputs):
            raise ValueError(f"expected {len(self.inputs)} inputs, got {len(host_inputs)}")
        if not hasattr(self, "_loss_host"):
            self._loss_host = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]
            self._loss_ev = [torch.cuda.Event(), torch.cuda.Event()]
            self._slot = 0
            self._pending = False
        for dst, src in zip(self.inputs, host_inputs):
            dst.copy_(src, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            loss = self.graph_loss
        else:
            loss = self.step_fn()
        prev = self._slot
        self._slot ^= 1
        self._loss_host[self._slot].copy_(loss.detach().reshape(()).float(), non_blocking=True)
        self._loss_ev[self._slot].record()
        out = None
        if self._pending:
            self._loss_ev[prev].synchronize()
            out = float(self._loss_host[prev])
        self._pending = True
        return out

    def flush(self) -> Optional[float]:
        """Loss of the last ``step_pipelined`` call (waits for it)."""
        if not getattr(self, "_pending", False):
            return None
        self._loss_ev[self._slot].synchronize()
        self._pending = False
        return float(self._loss_host[self._slot])
