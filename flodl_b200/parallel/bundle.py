"""Checkpoint bundle: ``<stem>.fdl`` (model) + ``<stem>.optim`` (optimizer
state) + ``<stem>.meta.json`` (training metadata, schema v5) + optional
``<stem>.outer.fdl`` (outer-optimizer state).

Reference: flodl/src/distributed/checkpoint_meta.rs:1-60,253-462 and
checkpoint_forge.rs (bundles are written atomically; a bundle is valid only
when all of its files exist).
"""
from __future__ import annotations

import json
import os
import time
from typing import Optional

import torch

from ..nn.checkpoint import load_model, save_checkpoint, save_model

META_SCHEMA = 5


def _atomic_json(path: str, obj: dict) -> None:
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        json.dump(obj, f, indent=2, sort_keys=True)
    os.replace(tmp, path)


def save_bundle(stem: str, model, optimizer=None, meta: Optional[dict] = None,
                outer_state: Optional[torch.Tensor] = None, reason: str = "periodic") -> None:
    save_model(model, stem + ".fdl")
    if optimizer is not None and hasattr(optimizer, "save_state_file"):
        optimizer.save_state_file(stem + ".optim")
    if outer_state is not None:
        save_checkpoint(stem + ".outer.fdl", [("outer/velocity", outer_state.detach().cpu())])
    m = {"schema": META_SCHEMA, "saved_at": time.time(), "reason": reason}
    m.update(meta or {})
    _atomic_json(stem + ".meta.json", m)


def load_bundle(stem: str, model, optimizer=None) -> dict:
    with open(stem + ".meta.json") as f:
        meta = json.load(f)
    if meta.get("schema", 0) > META_SCHEMA:
        raise ValueError(f"{stem}.meta.json: schema {meta.get('schema')} is newer than supported")
    load_model(model, stem + ".fdl")
    if optimizer is not None and os.path.exists(stem + ".optim"):
        optimizer.load_state_file(stem + ".optim")
    return meta


def bundle_complete(stem: str) -> bool:
    return all(os.path.exists(stem + s) for s in (".fdl", ".meta.json"))
