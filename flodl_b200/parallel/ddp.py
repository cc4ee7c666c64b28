"""Classic per-step data parallelism: the ``Ddp`` bypass tier.

Reference: flodl/src/distributed/ddp.rs:67-360 (``Ddp::wrap``, ``sync_params``,
``all_reduce_gradients`` (Avg), ``weighted_all_reduce_gradients``,
``sync_buffers``, ``average_params``). The reference all-reduces every gradient
in one grouped NCCL call after backward. Here gradients live in one flat f32
arena (shared with the optimizer) cut into buckets in reverse parameter order;
each bucket is reduced as soon as the fused backward reports all its
parameters ready, on a communication stream that overlaps the rest of
backward. Two engines:

* ``"nccl"``  one ``all_reduce`` (Avg) per bucket through torch.distributed
  (the measured baseline).
* ``"peer"``  the peer-memory communicator: one sm_100a kernel per bucket that
  reduce-scatters the bucket over NVLink by peer loads, applies the optimizer
  update to its shard and writes the updated parameters into every peer's
  arena (fused all-reduce + AdamW/SGD, see ``flodl_b200.parallel.fused``).
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Sequence

import torch
import torch.distributed as dist

from ..utils import log

from ..ops._common import add_grad_ready_listener, clear_grad_ready_listeners
from ..utils.arena import ParamArena, arena_of


class Bucket:
    __slots__ = ("start", "end", "params", "pending", "index")

    def __init__(self, index: int, start: int, end: int, params):
        self.index = index
        self.start, self.end = start, end
        self.params = list(params)
        self.pending = len(self.params)


class Ddp:
    """Wraps a model for per-step gradient all-reduce (world size from the
    default process group)."""

    def __init__(self, model: torch.nn.Module, bucket_mb: float = 25.0, engine: str = "nccl",
                 group=None, broadcast: bool = True):
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.engine = engine
        params = [p for p in model.parameters() if p.requires_grad]
        self.params = params
        self.device = params[0].device
        self.arena = arena_of(params) or ParamArena(params)
        self.comm_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self._build_buckets(bucket_mb)
        self._launched: List[Bucket] = []
        self.overlap = True
        for p in params:
            clear_grad_ready_listeners(p)
            add_grad_ready_listener(p, self._on_ready)
        self._pidx = {id(p): i for i, p in enumerate(params)}
        if broadcast and self.world > 1:
            self.sync_params()

    @classmethod
    def wrap(cls, model, **kw) -> "Ddp":
        return cls(model, **kw)

    # ------------------------------------------------------------ buckets
    def _build_buckets(self, bucket_mb: float) -> None:
        cap = int(bucket_mb * (1 << 20) / 4)
        a = self.arena
        order = list(range(len(a.params)))[::-1]  # backward produces grads last-layer first
        self.buckets: List[Bucket] = []
        self._bucket_of: Dict[int, Bucket] = {}
        cur: List[int] = []
        size = 0
        for i in order:
            cur.append(i)
            size += a.params[i].numel()
            if size >= cap:
                self._close_bucket(cur)
                cur, size = [], 0
        if cur:
            self._close_bucket(cur)

    def _close_bucket(self, idx: List[int]) -> None:
        a = self.arena
        start = min(a.offsets[i] for i in idx)
        last = max(idx)
        end = a.offsets[last] + a.params[last].numel()
        end = min(((end + 63) // 64) * 64, a.numel)
        if idx[0] == len(a.params) - 1:
            end = a.numel
        b = Bucket(len(self.buckets), start, end, [a.params[i] for i in idx])
        self.buckets.append(b)
        for i in idx:
            self._bucket_of[id(a.params[i])] = b

    def reset_pending(self) -> None:
        for b in self.buckets:
            b.pending = len(b.params)
        self._launched = []

    def _on_ready(self, p: torch.Tensor) -> None:
        if self.world == 1 or not self.overlap:
            return
        b = self._bucket_of.get(id(p))
        if b is None:
            return
        b.pending -= 1
        if b.pending == 0:
            self._launch(b)

    def _launch(self, b: Bucket) -> None:
        cur = torch.cuda.current_stream(self.device)
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            sl = self.arena.grad[b.start:b.end]
            with log.collective("ddp.bucket_all_reduce", numel=sl.numel()):
                dist.all_reduce(sl, op=dist.ReduceOp.AVG, group=self.group)
        self._launched.append(b)

    # ------------------------------------------------------------ public API
    def all_reduce_gradients(self) -> None:
        """Finish the gradient average: launch buckets not yet launched (e.g.
        parameters without a fused-backward notification) and join the
        communication stream into the compute stream."""
        if self.world == 1:
            self.reset_pending()
            return
        if not self.overlap:
            with log.collective("ddp.all_reduce_gradients", numel=self.arena.grad.numel()):
                dist.all_reduce(self.arena.grad, op=dist.ReduceOp.AVG, group=self.group)
            self.reset_pending()
            return
        for b in self.buckets:
            if b not in self._launched:
                self._launch(b)
        torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)
        self.reset_pending()

    finish = all_reduce_gradients

    @torch.no_grad()
    def weighted_all_reduce_gradients(self, batch_counts: Sequence[float]) -> None:
        """Scale local grads by this rank's share of ``batch_counts`` then Sum."""
        total = float(sum(batch_counts))
        self.arena.grad.mul_(batch_counts[self.rank] / total)
        dist.all_reduce(self.arena.grad, op=dist.ReduceOp.SUM, group=self.group)
        self.reset_pending()

    @torch.no_grad()
    def sync_params(self) -> None:
        """Broadcast rank 0's parameters and buffers to every rank."""
        with log.collective("ddp.sync_params", numel=self.arena.data.numel()):
            dist.broadcast(self.arena.data, src=0, group=self.group)
        self.arena.refresh_shadow()
        self.sync_buffers()

    @torch.no_grad()
    def sync_buffers(self) -> None:
        for b in self.model.buffers():
            if b.is_floating_point():
                dist.broadcast(b, src=0, group=self.group)

    @torch.no_grad()
    def average_params(self) -> None:
        with log.collective("ddp.average_params", numel=self.arena.data.numel()):
            dist.all_reduce(self.arena.data, op=dist.ReduceOp.AVG, group=self.group)
        self.arena.refresh_shadow()

    @torch.no_grad()
    def all_reduce_per_rank_f64(self, value: float) -> List[float]:
        t = torch.zeros(self.world, dtype=torch.float64, device=self.device)
        t[self.rank] = value
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t.tolist()


def init_from_env(backend: Optional[str] = None, timeout_s: float = 120.0):
    """Initialise torch.distributed from torchrun's environment (idempotent).
    Returns (rank, world, local_rank)."""
    import datetime

    if "RANK" not in os.environ or int(os.environ.get("WORLD_SIZE", "1")) <= 1:
        return 0, 1, int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return rank, world, local
