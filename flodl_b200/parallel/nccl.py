"""NCCL communicator layer: per-rank communicators, the single-process group
API, PreMulSum, broadcast and a thread-safe abort handle.

Reference: flodl/src/distributed/nccl.rs:36-787 (``ReduceOp``, ``NcclComms``
group init + ``split``, ``NcclUniqueId``, ``NcclAbortHandle``,
``NcclRankComm::init_rank``, ``all_reduce_premul_sum``, ``broadcast``).

Per-rank communicators ride ``torch.distributed`` process groups (NCCL on
CUDA tensors, gloo on CPU tensors, so the host-side logic tests on CPU). The
unique id is the rendezvous address the first rank picks - 128 bytes, like
NCCL's - and every rank initialises from it. ``NcclComms`` is the
single-process, multi-device group (one communicator per visible device)
through ``torch.cuda.nccl``'s grouped collectives. The framework's hot
collectives are its own peer-memory kernels (:mod:`flodl_b200.parallel.peer`);
this layer is the baseline and the bootstrap.
"""
from __future__ import annotations

import datetime
import enum
import json
import socket
import threading
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


class ReduceOp(enum.Enum):
    Sum = "sum"
    Avg = "avg"
    Max = "max"
    Min = "min"
    Prod = "prod"

    def torch(self):
        return {"sum": dist.ReduceOp.SUM, "avg": dist.ReduceOp.AVG, "max": dist.ReduceOp.MAX,
                "min": dist.ReduceOp.MIN, "prod": dist.ReduceOp.PRODUCT}[self.value]


UNIQUE_ID_BYTES = 128


class NcclUniqueId:
    """128 opaque bytes shared out of band (e.g. by the rendezvous)."""

    def __init__(self, raw: bytes):
        if len(raw) != UNIQUE_ID_BYTES:
            raise ValueError(f"a unique id is {UNIQUE_ID_BYTES} bytes")
        self.raw = raw

    @staticmethod
    def new(host: str = "127.0.0.1") -> "NcclUniqueId":
        s = socket.socket()
        s.bind((host, 0))
        port = s.getsockname()[1]
        s.close()
        body = json.dumps({"h": host, "p": port}).encode()
        return NcclUniqueId(body.ljust(UNIQUE_ID_BYTES, b"\0"))

    def address(self):
        d = json.loads(self.raw.rstrip(b"\0").decode())
        return d["h"], d["p"]


class NcclAbortHandle:
    """Thread-safe, idempotent abort of a communicator (unblocks ranks
    stuck in a collective with a dead peer)."""

    def __init__(self, comm: "NcclRankComm"):
        self._comm = comm
        self._lock = threading.Lock()
        self.aborted = False

    def abort(self) -> None:
        with self._lock:
            if self.aborted:
                return
            self.aborted = True
            self._comm._abort()


class NcclRankComm:
    """This process's communicator within a group of ``world`` ranks."""

    def __init__(self, group, rank: int, world: int, owns_default: bool):
        self.group, self.rank, self.world = group, rank, world
        self._owns_default = owns_default
        self.abort_handle = NcclAbortHandle(self)

    @staticmethod
    def init_rank(rank: int, world: int, uid: NcclUniqueId, device=None,
                  timeout_s: float = 120.0, backend: Optional[str] = None) -> "NcclRankComm":
        host, port = uid.address()
        dev = torch.device(device) if device is not None else torch.device("cpu")
        backend = backend or ("nccl" if dev.type == "cuda" else "gloo")
        kw = {"device_id": dev} if backend == "nccl" else {}
        if backend == "nccl":
            torch.cuda.set_device(dev)
        dist.init_process_group(backend, init_method=f"tcp://{host}:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=timeout_s), **kw)
        return NcclRankComm(None, rank, world, True)

    def split(self, color: int, key: Optional[int] = None) -> Optional["NcclRankComm"]:
        """Sub-communicator of the ranks that passed the same ``color``
        (every rank must call; ranks are ordered by ``key`` then rank)."""
        mine = [color, self.rank if key is None else key, self.rank]
        allv: List[Optional[list]] = [None] * self.world
        dist.all_gather_object(allv, mine, group=self.group)
        colors = sorted({c for c, _, _ in allv})
        mine_group = None
        for c in colors:  # every rank creates every group, in the same order
            members = [r for _, _, r in sorted((k, r, r) for cc, k, r in allv if cc == c)]
            g = dist.new_group(members)
            if c == color:
                mine_group = (g, members)
        if mine_group is None:
            return None
        g, members = mine_group
        return NcclRankComm(g, members.index(self.rank), len(members), False)

    # ------------------------------------------------------------ collectives
    def all_reduce(self, tensors: Sequence[torch.Tensor], op: ReduceOp = ReduceOp.Sum) -> None:
        works = [dist.all_reduce(t, op=op.torch(), group=self.group, async_op=True) for t in tensors]
        for w in works:
            w.wait()

    def all_reduce_premul_sum(self, tensors: Sequence[torch.Tensor], factor: float) -> None:
        """``sum_r factor_r * t_r`` in place (each rank passes its own factor)."""
        nccl = all(t.is_cuda for t in tensors) and dist.get_backend(self.group) == "nccl"
        if nccl and hasattr(dist, "_make_nccl_premul_sum"):
            op = dist._make_nccl_premul_sum(float(factor))
            works = [dist.all_reduce(t, op=op, group=self.group, async_op=True) for t in tensors]
        else:
            for t in tensors:
                t.mul_(factor)
            works = [dist.all_reduce(t, group=self.group, async_op=True) for t in tensors]
        for w in works:
            w.wait()

    def broadcast(self, tensors: Sequence[torch.Tensor], root: int = 0) -> None:
        src = root if self.group is None else dist.get_global_rank(self.group, root)
        works = [dist.broadcast(t, src, group=self.group, async_op=True) for t in tensors]
        for w in works:
            w.wait()

    def all_reduce_per_rank_f64(self, value: float) -> List[float]:
        """Every rank's value (the timing exchange)."""
        t = torch.zeros(self.world, dtype=torch.float64)
        dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(self.group) == "nccl" else "cpu"
        t = t.to(dev)
        t[self.rank] = value
        dist.all_reduce(t, group=self.group)
        return t.cpu().tolist()

    def _abort(self) -> None:
        try:
            g = self.group or dist.distributed_c10d._get_default_group()
            backend = g._get_backend(torch.device("cuda")) if torch.cuda.is_available() else None
            if backend is not None and hasattr(backend, "abort"):
                backend.abort()
        except Exception:
            pass

    def close(self) -> None:
        if self._owns_default and dist.is_initialized():
            dist.destroy_process_group()


class NcclComms:
    """Single-process group over several devices (one rank per device),
    with grouped collectives over lists of per-device tensors."""

    def __init__(self, devices: Sequence[int]):
        import torch.cuda.nccl as tnccl
        self.nccl = tnccl
        self.devices = list(devices)

    def all_reduce(self, tensors: Sequence[torch.Tensor], op: ReduceOp = ReduceOp.Sum) -> None:
        if op is ReduceOp.Avg:
            self.nccl.all_reduce(list(tensors))
            for t in tensors:
                t.div_(len(tensors))
            return
        code = {ReduceOp.Sum: 0, ReduceOp.Prod: 1, ReduceOp.Max: 2, ReduceOp.Min: 3}[op]
        self.nccl.all_reduce(list(tensors), op=code)

    def broadcast(self, tensors: Sequence[torch.Tensor], root: int = 0) -> None:
        self.nccl.broadcast(list(tensors), root=root)

    def split(self) -> List["NcclComms"]:
        """One single-device view per device (the per-thread communicators)."""
        return [NcclComms([d]) for d in self.devices]

    @staticmethod
    def version() -> str:
        v = torch.cuda.nccl.version()
        return ".".join(map(str, v)) if isinstance(v, tuple) else str(v)
