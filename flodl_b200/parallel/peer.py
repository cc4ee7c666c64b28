"""Peer-memory communicator (single node, NVLink 5 / NVSwitch).

Replaces the reference's NCCL communicator layer (flodl/src/distributed/nccl.rs)
for the hot collectives. Each rank allocates symmetric regions with
``cudaMalloc`` and exports CUDA IPC handles; the handles are exchanged once
over the torch.distributed process group (NCCL or gloo — bootstrap only);
every rank maps its peers' regions, so the fused sm_100a kernels in
``peer_comm.cu`` load from and store to any rank's memory directly.

Regions per communicator: ``data`` (f32), ``grad`` (f32), ``shadow`` (bf16,
optional) of ``numel`` elements, and the signal words. Waits inside the
kernels are bounded; a timeout sets a word in host-mapped memory that
:meth:`PeerComm.check` turns into an exception, and the communicator is then
unusable (the caller rebuilds it, as the reference does after
``ncclCommAbort``).
"""
from __future__ import annotations

from typing import List, Optional

import torch

from ..utils import log
import torch.distributed as dist

from .._ext import cuda_ext

ERR_NAMES = {1: "mbarrier wait timed out", 2: "peer wait timed out", 3: "bad arguments"}


class PeerTimeout(RuntimeError):
    pass


class PeerComm:
    """Symmetric peer-mapped buffers of one rank plus the fused collective
    launches over them. ``blocks`` arguments: CTAs per launch, 0 = as many as
    can be co-resident (the kernels wait on all of their own blocks)."""

    def __init__(self, numel: int, device: torch.device, group=None, with_shadow: bool = True,
                 timeout_s: float = 10.0):
        C = cuda_ext()
        self.C = C
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if self.world > C.MAX_RANKS:
            raise ValueError(f"PeerComm supports up to {C.MAX_RANKS} ranks on one node")
        self.device = torch.device(device)
        self.numel = (numel + 63) // 64 * 64
        self.timeout_ns = int(timeout_s * 1e9)
        self._own: List[int] = []
        self._opened: List[int] = []
        sig_words = C.signal_words()
        regions = [("data", self.numel * 4), ("grad", self.numel * 4)]
        if with_shadow:
            regions.append(("shadow", self.numel * 2))
        regions.append(("sig", sig_words * 4))
        local = {}
        handles = {}
        with torch.cuda.device(self.device):
            for name, nbytes in regions:
                ptr, h = C.peer_alloc(nbytes)
                self._own.append(ptr)
                local[name] = ptr
                handles[name] = h
        gathered: List[Optional[dict]] = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(gathered, handles, group=self.group)
        else:
            gathered = [handles]
        self.ptrs = {name: [0] * self.world for name, _ in regions}
        with torch.cuda.device(self.device):
            for p in range(self.world):
                for name, _ in regions:
                    if p == self.rank:
                        self.ptrs[name][p] = local[name]
                    else:
                        ptr = C.peer_open(gathered[p][name])
                        self._opened.append(ptr)
                        self.ptrs[name][p] = ptr
        dev = self.device.index
        self.data = C.tensor_from_ptr(local["data"], self.numel, "float32", dev)
        self.grad = C.tensor_from_ptr(local["grad"], self.numel, "float32", dev)
        self.shadow = (C.tensor_from_ptr(local["shadow"], self.numel, "bfloat16", dev)
                       if with_shadow else None)
        if not with_shadow:
            self.ptrs["shadow"] = [0] * self.world
        self.err_host, self.err_dev = C.host_mapped_words(4)
        self.closed = False

    # ------------------------------------------------------------ allocators for ParamArena
    def data_alloc(self, n, dtype, device):
        assert n <= self.numel and dtype == torch.float32
        return self.data[:n]

    def grad_alloc(self, n, dtype, device):
        assert n <= self.numel and dtype == torch.float32
        return self.grad[:n]

    # ------------------------------------------------------------ launches
    def launch(self, op: int, **cfg) -> None:
        if self.closed:
            raise RuntimeError("PeerComm used after close/abort")
        cfg.setdefault("rank", self.rank)
        cfg.setdefault("world", self.world)
        cfg.setdefault("timeout_ns", self.timeout_ns)
        cfg.setdefault("err", self.err_dev)
        with log.collective("peer.fused_launch", op=op, bucket=cfg.get("bucket", 0),
                            start=cfg.get("start", 0), end=cfg.get("end", 0)):
            self.C.fused_launch(op, cfg, self.ptrs["data"], self.ptrs["grad"], self.ptrs["shadow"],
                                self.ptrs["sig"])

    def check(self) -> None:
        """Raise if a kernel recorded a timeout (no device synchronisation)."""
        code = int(self.err_host[0].item())
        if code:
            raise PeerTimeout(f"peer communicator: {ERR_NAMES.get(code, code)} on rank {self.rank}")

    def all_reduce_(self, n: int, average: bool = True, slot: int = 0, blocks: int = 0,
                    oneshot: bool = False, threads: int = 512) -> None:
        """In-place all-reduce of grad[:n]. The one-shot form reads every
        peer's whole range and uses data[:n] as scratch."""
        self.launch(self.C.FUSED_ALL_REDUCE, bucket=slot, start=0, end=(n + 3) // 4 * 4,
                    average=int(average), blocks=blocks, oneshot=int(oneshot), threads=threads)

    def broadcast_(self, n: int, root: int = 0, slot: int = 0, blocks: int = 0) -> None:
        """Every rank pulls data[:n] (and refreshes its bf16 shadow) from ``root``."""
        self.launch(self.C.FUSED_BROADCAST, bucket=slot, start=0, end=(n + 3) // 4 * 4, root=root,
                    blocks=blocks)

    def weighted_average_(self, n: int, mass: float, slot: int = 0,
                          div: Optional[torch.Tensor] = None, blocks: int = 0,
                          mover: Optional[float] = None, buf_start: int = -1) -> None:
        """Cluster averaging over data[:n] (flodl/src/distributed/ddp_run/worker/
        sync.rs:130-236): data[:buf_start] <- sum_i (mass_i / sum mass) data_i
        (``mass`` is this rank's gamma-mass n^gamma, 0 for an idle rank) and
        data[buf_start:n] (f32 buffers) <- mean over the ranks that did work
        (``mover``, default 1 if mass > 0). Nothing changes when no rank did
        work. ``div`` (f32 [2], zeroed by the caller) receives this rank's
        ||pre - post||^2 and ||post||^2 over the parameter part."""
        if mover is None:
            mover = 1.0 if mass > 0 else 0.0
        if buf_start >= 0 and buf_start % 4:
            raise ValueError("buf_start must be a multiple of 4 elements")
        self.launch(self.C.FUSED_WEIGHTED_AVG, bucket=slot, start=0, end=(n + 3) // 4 * 4,
                    mass=float(mass), mover=float(mover), buf_start=int(buf_start), div=div,
                    blocks=blocks)

    def close(self) -> None:
        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                try:
                    self.C.peer_close(p)
                except Exception:
                    pass
        self._opened = []
        # own regions are freed last, after every peer closed its mapping
        if self.world > 1 and dist.is_initialized():
            try:
                dist.barrier(group=self.group)
            except Exception:
                pass
        with torch.cuda.device(self.device):
            for p in self._own:
                try:
                    self.C.peer_free(p)
                except Exception:
                    pass
        self._own = []
        self.closed = True

    abort = close

    def abandon(self) -> None:
        """Give the communicator up without any peer: waits for this rank's
        own work, unmaps the peers' regions and frees this rank's regions. No
        kernel touches a peer's memory again and no collective runs, so this
        is safe after a peer left or died (survivor re-formation)."""
        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                try:
                    self.C.peer_close(p)
                except Exception:
                    pass
            for p in self._own:
                try:
                    self.C.peer_free(p)
                except Exception:
                    pass
        self._opened, self._own = [], []
        self.closed = True
