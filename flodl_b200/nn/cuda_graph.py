"""CUDA graph capture/replay (flodl/src/nn/cuda_graph.rs:85-164).

``GpuGraph`` captures a callable once on a side stream (after warm-up) and
replays it; static input/output tensors are reused between replays. This is
how the training engine removes per-kernel launch overhead from whole steps.
"""
from __future__ import annotations

import enum
from typing import Callable, Optional

import torch


class CaptureMode(enum.Enum):
    GLOBAL = "global"
    THREAD_LOCAL = "thread_local"
    RELAXED = "relaxed"


class MemPoolId(tuple):
    pass


def gpu_graph_pool_handle():
    return torch.cuda.graph_pool_handle()


class GpuGraph:
    def __init__(self, pool=None, mode: CaptureMode = CaptureMode.THREAD_LOCAL):
        self.graph = torch.cuda.CUDAGraph()
        self.pool = pool
        self.mode = mode
        self.output = None
        self.captured = False

    def capture(self, fn: Callable, warmup: int = 2):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        # capture on the warm-up stream: autograd nodes that outlive a warm-up
        # step (e.g. loop traces kept for inspection) carry that stream, and a
        # backward that touches them from another stream would wait on work
        # outside the capture
        with torch.cuda.graph(self.graph, pool=self.pool, stream=s,
                              capture_error_mode=self.mode.value):
            self.output = fn()
        self.captured = True
        return self.output

    def replay(self):
        if not self.captured:
            raise RuntimeError("GpuGraph.replay() before capture()")
        self.graph.replay()
        return self.output

    def reset(self):
        self.graph.reset()
        self.captured = False
        self.output = None

    def pool_id(self):
        return self.graph.pool()


def gpu_graph_capture(fn: Callable, warmup: int = 2, pool=None) -> GpuGraph:
    g = GpuGraph(pool)
    g.capture(fn, warmup)
    return g
