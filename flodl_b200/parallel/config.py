"""Distributed training configuration (flodl/src/distributed/config.rs:58-990).

``ElCheMode`` = (apply policy, averaging backend):

    NcclSync    (Sync,    peer-memory/NCCL)  average after every step window of 1
    NcclCadence (Cadence, peer-memory/NCCL)  ElChe windows, then weighted average (default)
    CpuSync     (Sync,    CPU reducer)
    CpuCadence  (Cadence, CPU reducer)
    CpuAsync    (Async,   CPU reducer)       bounded overshoot + EASGD blend

(Async, device backend) has no mode, as in floDl. The "Nccl" names are kept
for API parity; on one NVLink node the device backend is the peer-memory
communicator's fused averaging kernel.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import Callable, List, Optional


class ApplyPolicy(enum.Enum):
    SYNC = "sync"
    CADENCE = "cadence"
    ASYNC = "async"


class AverageBackend(enum.Enum):
    NCCL = "nccl"
    CPU = "cpu"


class ElCheMode(enum.Enum):
    NcclSync = "nccl-sync"
    NcclCadence = "nccl-cadence"
    CpuSync = "cpu-sync"
    CpuCadence = "cpu-cadence"
    CpuAsync = "cpu-async"

    def split(self):
        return {
            ElCheMode.NcclSync: (ApplyPolicy.SYNC, AverageBackend.NCCL),
            ElCheMode.NcclCadence: (ApplyPolicy.CADENCE, AverageBackend.NCCL),
            ElCheMode.CpuSync: (ApplyPolicy.SYNC, AverageBackend.CPU),
            ElCheMode.CpuCadence: (ApplyPolicy.CADENCE, AverageBackend.CPU),
            ElCheMode.CpuAsync: (ApplyPolicy.ASYNC, AverageBackend.CPU),
        }[self]

    @staticmethod
    def from_parts(policy: ApplyPolicy, backend: AverageBackend) -> "ElCheMode":
        for m in ElCheMode:
            if m.split() == (policy, backend):
                return m
        raise ValueError("(Async, Nccl) has no ElCheMode")


@dataclass
class ElCheConfig:
    mode_: ElCheMode = ElCheMode.NcclCadence
    anchor_: int = 10
    max_anchor_: int = 0
    min_anchor_: int = 1
    overhead_target_: float = 0.05
    max_batch_diff_: int = 0
    relax_up_: bool = False
    partition_ratios_: Optional[List[float]] = None
    meta_controller_: bool = True
    easgd_alpha_: float = 0.5
    divergence_threshold_: float = 0.05
    divergence_guard_: bool = True
    max_overshoot_: int = 3
    gamma_: float = 1.0

    # chained setters with floDl's names
    def mode(self, m: ElCheMode):
        self.mode_ = m
        return self

    def anchor(self, n: int):
        self.anchor_ = n
        return self

    def max_anchor(self, n: int):
        self.max_anchor_ = n
        return self

    def min_anchor(self, n: int):
        self.min_anchor_ = n
        return self

    def overhead_target(self, f: float):
        self.overhead_target_ = f
        return self

    def max_batch_diff(self, n: int):
        self.max_batch_diff_ = n
        return self

    def relax_up(self, on: bool):
        self.relax_up_ = on
        return self

    def partition_ratios(self, r: List[float]):
        self.partition_ratios_ = list(r)
        return self

    def meta_controller(self, on: bool):
        self.meta_controller_ = on
        return self

    def easgd_alpha(self, a: float):
        self.easgd_alpha_ = a
        return self

    def divergence_threshold(self, t: float):
        self.divergence_threshold_ = t
        return self

    def no_divergence_guard(self):
        self.divergence_guard_ = False
        return self

    def max_overshoot(self, n: int):
        self.max_overshoot_ = n
        return self

    def gamma(self, g: float):
        self.gamma_ = g
        return self

    @classmethod
    def sync(cls):
        return cls(mode_=ElCheMode.NcclSync, anchor_=1)

    @classmethod
    def cadence(cls):
        return cls(mode_=ElCheMode.NcclCadence)


@dataclass
class TrainerConfig:
    batch_size_: int = 32
    num_epochs_: int = 1
    elche_: ElCheConfig = field(default_factory=ElCheConfig)
    max_grad_norm_: Optional[float] = None
    checkpoint_every_: int = 0
    save_path_: Optional[str] = None
    resume_from_: Optional[str] = None
    eval_every_: int = 0
    reports_per_epoch_: int = 1
    heartbeat_timeout_secs_: float = 30.0
    record_log_: Optional[str] = None
    epoch_fn_: Optional[Callable] = None
    eval_fn_: Optional[Callable] = None
    scheduler_fn_: Optional[Callable] = None
    metrics_fn_: Optional[Callable] = None
    checkpoint_fn_: Optional[Callable] = None

    def batch_size(self, n):
        self.batch_size_ = n
        return self

    def num_epochs(self, n):
        self.num_epochs_ = n
        return self

    def elche(self, cfg: ElCheConfig):
        self.elche_ = cfg
        return self

    def max_grad_norm(self, n):
        self.max_grad_norm_ = n
        return self

    def checkpoint_every(self, n):
        self.checkpoint_every_ = n
        return self

    def save_path(self, p):
        self.save_path_ = p
        return self

    def resume_from(self, p):
        self.resume_from_ = p
        return self

    def eval_every(self, n):
        self.eval_every_ = n
        return self

    def reports_per_epoch(self, n):
        self.reports_per_epoch_ = n
        return self

    def heartbeat_timeout_secs(self, s):
        self.heartbeat_timeout_secs_ = s
        return self

    def record_log(self, path):
        self.record_log_ = path
        return self

    def epoch_fn(self, f):
        self.epoch_fn_ = f
        return self

    def eval_fn(self, f):
        self.eval_fn_ = f
        return self

    def scheduler_fn(self, f):
        self.scheduler_fn_ = f
        return self

    def metrics_fn(self, f):
        self.metrics_fn_ = f
        return self

    def checkpoint_fn(self, f):
        self.checkpoint_fn_ = f
        return self
