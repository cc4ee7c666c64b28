"""Cluster topology: per-rank envelope, builder, model signature, test discovery.

Reference roles:

* :class:`LocalCluster` - the slim per-node envelope a launcher ships to each
  rank in ``FLODL_INTERNAL_CLUSTER_JSON`` (flodl/src/distributed/cluster.rs:
  150-560): controller address, world size, this worker's ranks and devices.
  The JSON field names are the reference's (``controller.host/port``,
  ``world_size``, ``num_workers``, ``worker.{host, ranks, local_devices,
  nccl_socket_ifname, path, arch, data_path, gpu_ram_share}``, ``salt``,
  ``rank_resources``) so envelopes written by either launcher parse here.
* :class:`ClusterBuilder` / :class:`HostBuilder` -> :class:`FullCluster` - the
  launcher-side topology (cluster_builder.rs:56-640, launcher/types.rs:79):
  ranks across hosts must form ``0..world`` without gaps or duplicates,
  devices and ranks pair one to one, launcher-owned env keys are reserved.
* :func:`model_sig` - SHA-256 over the parameter and buffer manifest in
  declaration order (model_sig.rs): ranks with unequal signatures must not
  average each other's parameters, so formation refuses a mismatch.
* :func:`discover_test_cluster` - tests find a topology in
  ``FLODL_TESTING_CLUSTER_JSON`` (hex-encoded JSON) or synthesise a loopback
  cluster with one rank per visible device (testing.rs:56).
"""
from __future__ import annotations

import json
import os
import socket
import struct
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch

ENV_CLUSTER_JSON = "FLODL_INTERNAL_CLUSTER_JSON"
ENV_FULL_CLUSTER_JSON = "FLODL_INTERNAL_FULL_CLUSTER_JSON"
ENV_HOST_OVERRIDE = "FLODL_HOST_NAME"
ENV_LOCAL_RANK = "FLODL_INTERNAL_LOCAL_RANK"
ENV_TESTING_CLUSTER_JSON = "FLODL_TESTING_CLUSTER_JSON"
ENV_FDL_ENV = "FDL_ENV"
SALT_BYTES = 16

_RESERVED = {"CUDA_VISIBLE_DEVICES", "CUDA_DEVICE_ORDER", "HIP_VISIBLE_DEVICES",
             "ROCR_VISIBLE_DEVICES", "GPU_DEVICE_ORDINAL", ENV_HOST_OVERRIDE, ENV_FDL_ENV}


class ClusterError(ValueError):
    pass


def is_reserved_cluster_env_key(key: str) -> bool:
    """Env keys the launcher sets per rank; a cluster or host env block that
    set them would override the launcher's value."""
    return key.startswith("FLODL_INTERNAL_") or key in _RESERVED


def resolve_hostname(env=None) -> str:
    env = os.environ if env is None else env
    return env.get(ENV_HOST_OVERRIDE) or socket.gethostname()


# ----------------------------------------------------------------- per-rank envelope
@dataclass
class WorkerBlock:
    host: str
    ranks: List[int]
    local_devices: List[int]
    nccl_socket_ifname: str = ""
    path: str = "."
    arch: Optional[str] = None
    data_path: Optional[str] = None
    gpu_ram_share: Optional[float] = None

    def to_json(self) -> dict:
        return {"host": self.host, "ranks": self.ranks, "local_devices": self.local_devices,
                "nccl_socket_ifname": self.nccl_socket_ifname, "path": self.path,
                "arch": self.arch, "data_path": self.data_path,
                "gpu_ram_share": self.gpu_ram_share}


def _parse_worker(v) -> WorkerBlock:
    if not isinstance(v, dict):
        raise ClusterError("cluster: worker (object) required")
    host = v.get("host")
    if not isinstance(host, str) or not host.strip():
        raise ClusterError("cluster: worker.host (non-empty string) required")
    ranks = v.get("ranks")
    if not isinstance(ranks, list) or not ranks or not all(isinstance(r, int) and r >= 0 for r in ranks):
        raise ClusterError(f"cluster.worker ({host!r}): ranks must be a non-empty list of ints")
    devs = v.get("local_devices", "all")
    if devs == "all":
        devs = list(range(len(ranks)))
    if not isinstance(devs, list) or len(devs) != len(ranks):
        raise ClusterError(f"cluster.worker ({host!r}): local_devices ({devs}) must pair one "
                           f"to one with ranks ({ranks})")
    share = v.get("gpu_ram_share")
    if share is not None and not (isinstance(share, (int, float)) and share >= 0):
        raise ClusterError(f"cluster.worker ({host!r}): gpu_ram_share must be >= 0")
    return WorkerBlock(host, list(ranks), [int(d) for d in devs], v.get("nccl_socket_ifname", ""),
                       v.get("path", "."), v.get("arch"), v.get("data_path"), share)


@dataclass
class LocalCluster:
    controller_host: str
    controller_port: int
    world_size: int
    num_workers: int
    worker: WorkerBlock
    salt: bytes = bytes(SALT_BYTES)
    rank_resources: bool = False

    @staticmethod
    def from_value(v: dict) -> "LocalCluster":
        if not isinstance(v, dict):
            raise ClusterError("cluster: top-level JSON must be an object")
        c = v.get("controller")
        if not isinstance(c, dict):
            raise ClusterError("cluster: controller (object) required")
        host = c.get("host")
        if not isinstance(host, str) or not host.strip():
            raise ClusterError("cluster: controller.host must be non-empty")
        port = c.get("port")
        if not isinstance(port, int) or not 0 <= port < 65536:
            raise ClusterError("cluster: controller.port (u16) required")
        world = v.get("world_size")
        if not isinstance(world, int) or world <= 0:
            raise ClusterError("cluster: world_size must be > 0")
        nw = v.get("num_workers")
        if not isinstance(nw, int) or nw <= 0:
            raise ClusterError("cluster: num_workers must be > 0")
        if nw > world:
            raise ClusterError(f"cluster: num_workers ({nw}) cannot exceed world_size ({world})")
        w = _parse_worker(v.get("worker"))
        for r in w.ranks:
            if r >= world:
                raise ClusterError(f"cluster.worker ({w.host!r}): rank {r} out of bounds for "
                                   f"world_size {world}")
        salt = bytes(SALT_BYTES)
        if v.get("salt") is not None:
            salt = bytes.fromhex(v["salt"])
            if len(salt) != SALT_BYTES:
                raise ClusterError(f"cluster: salt must be {SALT_BYTES} bytes of hex")
        return LocalCluster(host, port, world, nw, w, salt, bool(v.get("rank_resources", False)))

    @staticmethod
    def from_json(path: str) -> "LocalCluster":
        with open(path) as f:
            return LocalCluster.from_value(json.load(f))

    @staticmethod
    def from_env(env=None) -> Optional["LocalCluster"]:
        env = os.environ if env is None else env
        raw = env.get(ENV_CLUSTER_JSON)
        if not raw:
            return None
        return LocalCluster.from_value(json.loads(raw))

    def to_json(self) -> dict:
        return {"controller": {"host": self.controller_host, "port": self.controller_port},
                "world_size": self.world_size, "num_workers": self.num_workers,
                "worker": self.worker.to_json(), "salt": self.salt.hex(),
                "rank_resources": self.rank_resources}

    def this_worker(self, env=None) -> WorkerBlock:
        name = resolve_hostname(env)
        if name != self.worker.host:
            raise ClusterError(f"cluster: resolved hostname {name!r} does not match the "
                               f"envelope's worker.host {self.worker.host!r} (set "
                               f"{ENV_HOST_OVERRIDE} to override on test rigs)")
        return self.worker

    def my_rank(self, env=None) -> Tuple[int, torch.device]:
        """(global rank, device). A single-value CUDA_VISIBLE_DEVICES means the
        child sees its one GPU as cuda:0."""
        env = os.environ if env is None else env
        w = self.this_worker(env)
        idx = int(env.get(ENV_LOCAL_RANK, env.get("LOCAL_RANK", "0")))
        if not 0 <= idx < len(w.ranks):
            raise ClusterError(f"cluster: local rank {idx} out of range for host {w.host!r} "
                               f"with {len(w.ranks)} ranks")
        vis = env.get("CUDA_VISIBLE_DEVICES", "")
        if vis and "," not in vis:
            return w.ranks[idx], torch.device("cuda", 0)
        return w.ranks[idx], torch.device("cuda", w.local_devices[idx])

    def spans_multiple_workers(self) -> bool:
        return self.num_workers > 1


# ----------------------------------------------------------------- launcher-side topology
@dataclass
class JoinKnobs:
    min_rank_start: Optional[int] = None
    join_timeout_secs: Optional[int] = None
    target_ranks: Optional[int] = None
    max_join_timeout_secs: Optional[int] = None
    open_admission: Optional[bool] = None
    discovery: Optional[bool] = None
    join_token: Optional[str] = None
    tunnel_only: Optional[bool] = None
    start_mode: Optional[str] = None


@dataclass
class FullController:
    host: str = ""
    port: int = 29500
    path: str = "."
    docker: Optional[str] = None
    arch: Optional[str] = None
    data_path: Optional[str] = None
    join: Optional[JoinKnobs] = None


@dataclass
class FullWorker:
    host: str
    ranks: List[int] = field(default_factory=list)
    local_devices: Optional[List[int]] = None       # None = all devices
    nccl_socket_ifname: str = ""
    path: Optional[str] = None
    arch: Optional[str] = None
    data_path: Optional[str] = None
    ssh: Optional[str] = None
    ssh_port: Optional[int] = None
    ssh_user: Optional[str] = None
    env: Dict[str, str] = field(default_factory=dict)
    gpu_ram_share: Optional[float] = None


@dataclass
class FullCluster:
    controller: FullController
    workers: List[FullWorker]
    salt: bytes = bytes(SALT_BYTES)
    env: Dict[str, str] = field(default_factory=dict)
    gpu_ram_share: Optional[float] = None

    @property
    def world_size(self) -> int:
        return sum(len(w.ranks) for w in self.workers)

    def with_session_salt(self, salt: Optional[bytes] = None) -> "FullCluster":
        self.salt = salt if salt is not None else os.urandom(SALT_BYTES)
        return self

    def envelope_for(self, host: str) -> LocalCluster:
        """The slim per-rank envelope of one worker host."""
        for w in self.workers:
            if w.host == host:
                devs = w.local_devices if w.local_devices is not None else list(range(len(w.ranks)))
                wb = WorkerBlock(w.host, list(w.ranks), list(devs), w.nccl_socket_ifname,
                                 w.path or self.controller.path, w.arch or self.controller.arch,
                                 w.data_path or self.controller.data_path,
                                 w.gpu_ram_share if w.gpu_ram_share is not None else self.gpu_ram_share)
                return LocalCluster(self.controller.host, self.controller.port, self.world_size,
                                    len(self.workers), wb, self.salt)
        raise ClusterError(f"cluster: no worker named {host!r}")

    def rank_env(self, host: str, local_index: int) -> Dict[str, str]:
        """Environment of one rank child: cluster env < host env < launcher keys."""
        w = next(w for w in self.workers if w.host == host)
        env = dict(self.env)
        env.update(w.env)
        env[ENV_CLUSTER_JSON] = json.dumps(self.envelope_for(host).to_json())
        env[ENV_LOCAL_RANK] = str(local_index)
        env[ENV_HOST_OVERRIDE] = host
        return env

    def to_json(self) -> dict:
        return {"controller": dict(self.controller.__dict__,
                                   join=self.controller.join.__dict__ if self.controller.join else None),
                "workers": [dict(w.__dict__) for w in self.workers], "salt": self.salt.hex(),
                "env": self.env, "gpu_ram_share": self.gpu_ram_share}

    @staticmethod
    def from_value(v: dict) -> "FullCluster":
        c = dict(v["controller"])
        join = c.pop("join", None)
        ctl = FullController(**c, join=JoinKnobs(**join) if join else None)
        workers = [FullWorker(**w) for w in v["workers"]]
        b = ClusterBuilder()
        b._controller, b._workers, b._env = ctl, workers, dict(v.get("env", {}))
        b._share = v.get("gpu_ram_share")
        fc = b.build()
        if v.get("salt"):
            fc.salt = bytes.fromhex(v["salt"])
        return fc


class ClusterBuilder:
    """Fluent topology builder, validated by :meth:`build`.

    ``ClusterBuilder().controller("ctl").port(29500).done()
       .host("a").ranks([0, 1]).devices([0, 1]).done()
       .host("b").ranks([2, 3]).all_devices().done().build()``
    """

    def __init__(self):
        self._controller = FullController()
        self._workers: List[FullWorker] = []
        self._env: Dict[str, str] = {}
        self._share: Optional[float] = None
        self._errors: List[str] = []

    def controller(self, host: str) -> "ControllerBuilder":
        self._controller.host = host
        return ControllerBuilder(self)

    def host(self, name: str) -> "HostBuilder":
        return HostBuilder(self, name)

    def env(self, key: str, value: str) -> "ClusterBuilder":
        self._env[key] = value
        return self

    def gpu_ram_share(self, share: float) -> "ClusterBuilder":
        self._share = share
        return self

    @staticmethod
    def all_local_gpus(port: int = 29500) -> FullCluster:
        from ..utils.hw import detect_gpus
        n = len(detect_gpus())
        if n == 0:
            raise ClusterError("ClusterBuilder.all_local_gpus: no GPU detected")
        return (ClusterBuilder().controller("127.0.0.1").port(port).done()
                .host("localhost").ranks(range(n)).all_devices().done().build())

    def build(self) -> FullCluster:
        if self._errors:
            raise ClusterError("ClusterBuilder: incomplete host definitions - " + "; ".join(self._errors))
        c = self._controller
        if not c.host.strip():
            raise ClusterError("ClusterBuilder: controller(...).done() needs a non-empty host")
        if not c.path.strip():
            raise ClusterError("ClusterBuilder: controller.path must be non-empty")
        discovery = bool(c.join and c.join.discovery)
        if not self._workers and not discovery:
            raise ClusterError("ClusterBuilder: at least one worker required (a roster-free "
                               "window needs discovery(True) on the controller)")
        for w in self._workers:
            if w.local_devices is not None and len(w.local_devices) != len(w.ranks):
                raise ClusterError(f"ClusterBuilder: host {w.host!r}: devices ({len(w.local_devices)}) "
                                   f"and ranks ({len(w.ranks)}) length mismatch")
        for k in self._env:
            if is_reserved_cluster_env_key(k):
                raise ClusterError(f"ClusterBuilder: cluster-scope env key {k!r} is reserved")
        for w in self._workers:
            for k in w.env:
                if is_reserved_cluster_env_key(k):
                    raise ClusterError(f"ClusterBuilder: host {w.host!r}: env key {k!r} is reserved")
        ok = lambda s: s is None or (s == s and s >= 0 and s != float("inf"))
        if not ok(self._share):
            raise ClusterError(f"ClusterBuilder: gpu_ram_share must be a non-negative fraction, "
                               f"got {self._share}")
        for w in self._workers:
            if not ok(w.gpu_ram_share):
                raise ClusterError(f"ClusterBuilder: host {w.host!r}: gpu_ram_share must be a "
                                   f"non-negative fraction, got {w.gpu_ram_share}")
        allr = sorted(r for w in self._workers for r in w.ranks)
        if allr != list(range(len(allr))):
            raise ClusterError(f"ClusterBuilder: ranks across workers must form 0..{len(allr)} with "
                               f"no duplicates or gaps, got {allr}")
        return FullCluster(c, list(self._workers), bytes(SALT_BYTES), dict(self._env), self._share)


class ControllerBuilder:
    def __init__(self, parent: ClusterBuilder):
        self.p = parent
        self.c = parent._controller

    def _join(self) -> JoinKnobs:
        if self.c.join is None:
            self.c.join = JoinKnobs()
        return self.c.join

    def port(self, port: int):
        self.c.port = port
        return self

    def path(self, p: str):
        self.c.path = p
        return self

    def docker(self, d: str):
        self.c.docker = d
        return self

    def arch(self, a: str):
        self.c.arch = a
        return self

    def data_path(self, p: str):
        self.c.data_path = p
        return self

    def min_rank_start(self, n: int):
        self._join().min_rank_start = n
        return self

    def join_timeout_secs(self, s: int):
        self._join().join_timeout_secs = s
        return self

    def target_ranks(self, n: int):
        self._join().target_ranks = n
        return self

    def max_join_timeout_secs(self, s: int):
        self._join().max_join_timeout_secs = s
        return self

    def open_admission(self, on: bool):
        self._join().open_admission = on
        return self

    def discovery(self, on: bool):
        self._join().discovery = on
        return self

    def join_token(self, hex_token: str):
        self._join().join_token = hex_token
        return self

    def tunnel_only(self, on: bool):
        self._join().tunnel_only = on
        return self

    def start_mode(self, mode):
        self._join().start_mode = getattr(mode, "value", mode)
        return self

    def done(self) -> ClusterBuilder:
        return self.p


class HostBuilder:
    def __init__(self, parent: ClusterBuilder, name: str):
        self.p = parent
        self.w = FullWorker(name)
        self._devices_set = False

    def ranks(self, ranks: Iterable[int]):
        self.w.ranks = list(ranks)
        return self

    def devices(self, devices: Iterable[int]):
        self.w.local_devices = list(devices)
        self._devices_set = True
        return self

    def all_devices(self):
        self.w.local_devices = None
        self._devices_set = True
        return self

    def nccl_socket_ifname(self, name: str):
        self.w.nccl_socket_ifname = name
        return self

    def path(self, p: str):
        self.w.path = p
        return self

    def arch(self, a: str):
        self.w.arch = a
        return self

    def data_path(self, p: str):
        self.w.data_path = p
        return self

    def ssh(self, target: str):
        self.w.ssh = target
        return self

    def ssh_port(self, port: int):
        self.w.ssh_port = port
        return self

    def ssh_user(self, user: str):
        self.w.ssh_user = user
        return self

    def env(self, key: str, value: str):
        self.w.env[key] = value
        return self

    def gpu_ram_share(self, s: float):
        self.w.gpu_ram_share = s
        return self

    def done(self) -> ClusterBuilder:
        if not self.w.ranks:
            self.p._errors.append(f"host {self.w.host!r}: ranks(...) not set")
        if not self._devices_set:
            self.p._errors.append(f"host {self.w.host!r}: devices(...) or all_devices() not set")
        self.p._workers.append(self.w)
        return self.p


# ----------------------------------------------------------------- model signature
def model_sig(params: Sequence[Tuple[str, torch.Tensor]],
              buffers: Sequence[Tuple[str, torch.Tensor]] = ()) -> bytes:
    """SHA-256 over (kind, name, dtype, shape) of every parameter then buffer,
    in declaration order (the averaging order), as 32 raw bytes."""
    from .._ext import native
    body = bytearray()
    for tag, items in ((b"P", params), (b"B", buffers)):
        for name, t in items:
            body += tag + name.encode() + b"\0"
            body += str(t.dtype).encode() + b"\0"
            body += struct.pack("<I", t.dim())
            for d in t.shape:
                body += struct.pack("<q", int(d))
    return bytes.fromhex(native().sha256_hex(bytes(body)))


def module_sig(module: torch.nn.Module) -> bytes:
    return model_sig(list(module.named_parameters()), list(module.named_buffers()))


# ----------------------------------------------------------------- test discovery
def discover_test_cluster(env=None) -> Optional[FullCluster]:
    """A topology for tests: ``FLODL_TESTING_CLUSTER_JSON`` (hex of the JSON),
    else a loopback cluster with one rank per visible CUDA device, else None.
    A malformed env value raises (a silent fallback would hide a bad config)."""
    env = os.environ if env is None else env
    raw = env.get(ENV_TESTING_CLUSTER_JSON)
    if raw:
        try:
            v = json.loads(bytes.fromhex(raw.strip()).decode())
        except (ValueError, UnicodeDecodeError) as e:
            raise ClusterError(f"{ENV_TESTING_CLUSTER_JSON}: not hex-encoded JSON: {e}") from e
        return FullCluster.from_value(v)
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n == 0:
        return None
    return (ClusterBuilder().controller("127.0.0.1").done()
            .host("localhost").ranks(range(n)).all_devices().done().build())
