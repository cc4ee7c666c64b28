"""Checkpoint bundle: ``<stem>.fdl`` (model) + ``<stem>.optim`` (optimizer
state) + ``<stem>.meta.json`` (training metadata) + optional
``<stem>.outer.fdl`` (outer-optimizer state) + per-rank
``<stem>.rank<N>.death.json`` records.

Reference: flodl/src/distributed/checkpoint_meta.rs (``CheckpointMeta``
schema v5, ``SaveReason``, ``ElCheState``, ``CoverageBlock``,
``RankDeathRecord``, ``CheckpointBundle`` paths) and checkpoint_forge.rs
(bundles written off the training thread, atomically).

``meta.json`` carries the reference's field names so bundles move between the
two frameworks: ``schema_version``, ``epoch``, ``global_step``, ``sync_round``,
``world_size_at_save``, ``save_reason`` (snake_case), ``elche_state`` (anchor,
anchor_rank, smoothed_ms_per_batch, phase, calibration_count, trend_history)
and ``coverage`` (seed, epoch_splits, batch_size, per_epoch: epoch,
total_samples, uncovered ``[offset, size]`` ranges of the epoch permutation).
Readers refuse a newer schema. Member paths replace one existing extension of
the stem (``ckpt.fdl`` and ``ckpt`` give the same bundle).
"""
from __future__ import annotations

import enum
import json
import os
import threading
import time
from dataclasses import asdict, dataclass, field
from typing import List, Optional, Tuple

import torch

from ..nn.checkpoint import load_model, save_checkpoint, save_model

CHECKPOINT_META_SCHEMA_VERSION = 5
RANK_DEATH_RECORD_SCHEMA_VERSION = 1
META_SCHEMA = CHECKPOINT_META_SCHEMA_VERSION


class SaveReason(enum.Enum):
    GracefulShutdown = "graceful_shutdown"
    MaxFailureExceeded = "max_failure_exceeded"
    SingleSurvivor = "single_survivor"
    AllRanksLost = "all_ranks_lost"
    ReduceStall = "reduce_stall"
    Checkpoint = "checkpoint"

    def to_u8(self) -> int:
        return list(SaveReason).index(self)

    @staticmethod
    def from_u8(b: int) -> Optional["SaveReason"]:
        members = list(SaveReason)
        return members[b] if 0 <= b < len(members) else None


@dataclass
class ElCheState:
    anchor: int
    anchor_rank: Optional[int]
    smoothed_ms_per_batch: List[float]
    phase: str = "probe"            # probe | warmup | stable | mature
    calibration_count: int = 0
    trend_history: Optional[List[float]] = None


@dataclass
class EpochCoverage:
    epoch: int
    total_samples: int
    uncovered_ranges: List[Tuple[int, int]]


@dataclass
class CoverageBlock:
    seed: int
    batch_size: int
    per_epoch: List[EpochCoverage] = field(default_factory=list)
    epoch_splits: int = 1


@dataclass
class CheckpointMeta:
    epoch: int
    global_step: int
    sync_round: int
    world_size_at_save: int
    save_reason: SaveReason = SaveReason.Checkpoint
    elche_state: Optional[ElCheState] = None
    coverage: Optional[CoverageBlock] = None
    schema_version: int = CHECKPOINT_META_SCHEMA_VERSION

    def to_json(self) -> dict:
        d = {"schema_version": self.schema_version, "epoch": self.epoch,
             "global_step": self.global_step, "sync_round": self.sync_round,
             "world_size_at_save": self.world_size_at_save, "save_reason": self.save_reason.value,
             "elche_state": asdict(self.elche_state) if self.elche_state else None,
             "coverage": None}
        if self.coverage is not None:
            c = self.coverage
            d["coverage"] = {"seed": c.seed, "epoch_splits": c.epoch_splits, "batch_size": c.batch_size,
                             "per_epoch": [{"epoch": e.epoch, "total_samples": e.total_samples,
                                            "uncovered_ranges": [list(r) for r in e.uncovered_ranges]}
                                           for e in c.per_epoch]}
        return d

    @staticmethod
    def from_json(d: dict, path: str = "meta.json") -> "CheckpointMeta":
        v = d.get("schema_version", 0)
        if v > CHECKPOINT_META_SCHEMA_VERSION:
            raise ValueError(f"CheckpointMeta: schema version {v} in {path} is newer than this "
                             f"build supports ({CHECKPOINT_META_SCHEMA_VERSION})")
        es = d.get("elche_state")
        cv = d.get("coverage")
        cov = None
        if cv:
            cov = CoverageBlock(cv["seed"], cv["batch_size"],
                                [EpochCoverage(e["epoch"], e["total_samples"],
                                               [tuple(r) for r in e["uncovered_ranges"]])
                                 for e in cv.get("per_epoch", [])], cv.get("epoch_splits", 1))
        return CheckpointMeta(d["epoch"], d.get("global_step", 0), d.get("sync_round", 0),
                              d.get("world_size_at_save", 1),
                              SaveReason(d.get("save_reason", "checkpoint")),
                              ElCheState(**es) if es else None, cov, v)


@dataclass
class RankDeathRecord:
    rank: int
    world_size: int
    error: str
    unix_time_secs: int = field(default_factory=lambda: int(time.time()))
    schema_version: int = RANK_DEATH_RECORD_SCHEMA_VERSION

    def write_to_file(self, path: str) -> None:
        _atomic_json(path, asdict(self))

    @staticmethod
    def read(path: str) -> "RankDeathRecord":
        with open(path) as f:
            return RankDeathRecord(**json.load(f))


def _with_ext(stem: str, ext: str) -> str:
    base, old = os.path.splitext(stem)
    if old and "/" not in old:
        stem = base
    return f"{stem}.{ext}"


class CheckpointBundle:
    model_path = staticmethod(lambda stem: _with_ext(stem, "fdl"))
    optim_path = staticmethod(lambda stem: _with_ext(stem, "optim"))
    meta_path = staticmethod(lambda stem: _with_ext(stem, "meta.json"))
    outer_path = staticmethod(lambda stem: _with_ext(stem, "outer.fdl"))
    config_sidecar_path = staticmethod(lambda stem: _with_ext(stem, "config.json"))

    @staticmethod
    def death_record_path(stem: str, rank: int) -> str:
        return _with_ext(stem, f"rank{rank}.death.json")


def _atomic_json(path: str, obj: dict) -> None:
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        json.dump(obj, f, indent=2, sort_keys=True)
    os.replace(tmp, path)


def save_bundle(stem: str, model, optimizer=None, meta=None,
                outer_state: Optional[torch.Tensor] = None, reason: str = "checkpoint") -> None:
    """Write the bundle; the meta file goes last, so a bundle whose
    ``meta.json`` exists is complete. ``meta`` is a :class:`CheckpointMeta`
    or a dict of its fields (``epoch`` required)."""
    save_model(model, CheckpointBundle.model_path(stem))
    if optimizer is not None and hasattr(optimizer, "save_state_file"):
        optimizer.save_state_file(CheckpointBundle.optim_path(stem))
    if outer_state is not None:
        save_checkpoint(CheckpointBundle.outer_path(stem), [("outer/velocity", outer_state.detach().cpu())])
    if not isinstance(meta, CheckpointMeta):
        d = dict(meta or {})
        meta = CheckpointMeta(d.get("epoch", 0), d.get("global_step", 0),
                              d.get("sync_round", d.get("syncs", 0)),
                              d.get("world_size_at_save", d.get("world", 1)),
                              SaveReason(d.get("save_reason", reason)),
                              d.get("elche_state"), d.get("coverage"))
    _atomic_json(CheckpointBundle.meta_path(stem), meta.to_json())


class CheckpointForge:
    """Writes bundles on a background thread (training continues); the
    model is copied to pinned host memory on a side stream first."""

    def __init__(self):
        self._threads: List[threading.Thread] = []
        self.errors: List[BaseException] = []

    def save(self, stem: str, model, optimizer=None, meta=None) -> threading.Thread:
        from ..graph.profile import ModelSnapshot
        snap = ModelSnapshot.take(model)
        opt_bytes = None
        if optimizer is not None and hasattr(optimizer, "save_state_file"):
            optimizer.save_state_file(CheckpointBundle.optim_path(stem) + ".tmp")
            opt_bytes = CheckpointBundle.optim_path(stem)

        def run():
            try:
                snap.save_file(CheckpointBundle.model_path(stem))
                if opt_bytes:
                    os.replace(opt_bytes + ".tmp", opt_bytes)
                m = meta if isinstance(meta, CheckpointMeta) else CheckpointMeta(**(meta or {"epoch": 0,
                    "global_step": 0, "sync_round": 0, "world_size_at_save": 1}))
                _atomic_json(CheckpointBundle.meta_path(stem), m.to_json())
            except BaseException as e:
                self.errors.append(e)

        t = threading.Thread(target=run, daemon=True)
        t.start()
        self._threads.append(t)
        return t

    def join(self) -> None:
        for t in self._threads:
            t.join()
        self._threads = []
        if self.errors:
            raise self.errors.pop(0)


def load_bundle(stem: str, model, optimizer=None) -> CheckpointMeta:
    path = CheckpointBundle.meta_path(stem)
    with open(path) as f:
        meta = CheckpointMeta.from_json(json.load(f), path)
    load_model(model, CheckpointBundle.model_path(stem))
    if optimizer is not None and os.path.exists(CheckpointBundle.optim_path(stem)):
        optimizer.load_state_file(CheckpointBundle.optim_path(stem))
    return meta


def read_meta(stem: str) -> CheckpointMeta:
    """The ``.meta.json`` of a bundle without loading any tensors."""
    path = CheckpointBundle.meta_path(stem)
    with open(path) as f:
        return CheckpointMeta.from_json(json.load(f), path)


def bundle_complete(stem: str) -> bool:
    return all(os.path.exists(p) for p in (CheckpointBundle.model_path(stem),
                                           CheckpointBundle.meta_path(stem)))
