"""`.fdl` checkpoints, byte-compatible with floDl (flodl/src/nn/checkpoint.rs).

The byte format is read and written by the native runtime
(``flodl_b200._native``: ``write_fdl``/``read_fdl``). Entries are matched by
qualified name; shape mismatches are errors; the structural hash (64 hex chars,
or all-zero to skip) is validated when both sides carry one.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .._ext import native


@dataclass
class LoadReport:
    loaded: List[str] = field(default_factory=list)
    skipped: List[str] = field(default_factory=list)
    missing: List[str] = field(default_factory=list)


@dataclass
class MigrateReport:
    renamed: List[Tuple[str, str]] = field(default_factory=list)
    unchanged: List[str] = field(default_factory=list)


def _named(model) -> Tuple[List[Tuple[str, torch.Tensor]], List[Tuple[str, torch.Tensor]]]:
    if hasattr(model, "graph_named_parameters"):
        return model.graph_named_parameters(), model.graph_named_buffers()
    params = [(n.replace(".", "/"), p) for n, p in torch.nn.Module.named_parameters(model)]
    bufs = [(n.replace(".", "/"), b) for n, b in torch.nn.Module.named_buffers(model)]
    return params, bufs


def save_checkpoint(path: str, params: Sequence[Tuple[str, torch.Tensor]],
                    buffers: Sequence[Tuple[str, torch.Tensor]] = (),
                    structural_hash: Optional[str] = None) -> None:
    entries = [(n, t.detach().cpu()) for n, t in list(params) + list(buffers)]
    native().write_fdl(path, entries, structural_hash)


save_checkpoint_file = save_checkpoint


def save_model(model, path: str) -> None:
    """Save a module/graph's parameters then buffers with its structural hash."""
    p, b = _named(model)
    h = model.structural_hash() if hasattr(model, "structural_hash") else None
    save_checkpoint(path, p, b, h)


def read_checkpoint(path: str):
    """(version, hash_hex, [(name, cpu tensor)]) of a `.fdl` file."""
    return native().read_fdl(path)


@torch.no_grad()
def load_checkpoint(path: str, params: Sequence[Tuple[str, torch.Tensor]],
                    buffers: Sequence[Tuple[str, torch.Tensor]] = (),
                    structural_hash: Optional[str] = None) -> LoadReport:
    _, fhash, entries = native().read_fdl(path)
    if structural_hash and any(c != "0" for c in fhash) and any(c != "0" for c in structural_hash):
        if fhash != structural_hash:
            raise ValueError(f"checkpoint architecture mismatch: file={fhash} model={structural_hash}")
    ck: Dict[str, torch.Tensor] = {n: t for n, t in entries}
    rep = LoadReport()
    for kind, items in (("parameter", params), ("buffer", buffers)):
        for name, t in items:
            src = ck.pop(name, None)
            if src is None:
                rep.missing.append(name)
                continue
            if tuple(src.shape) != tuple(t.shape):
                raise ValueError(f"{kind} {name!r}: shape mismatch: checkpoint={list(src.shape)} "
                                 f"model={list(t.shape)}")
            t.copy_(src.to(dtype=t.dtype, device=t.device))
            rep.loaded.append(name)
    rep.skipped = list(ck.keys())
    return rep


load_checkpoint_file = load_checkpoint


def load_model(model, path: str) -> LoadReport:
    p, b = _named(model)
    h = model.structural_hash() if hasattr(model, "structural_hash") else None
    rep = load_checkpoint(path, p, b, h)
    from ..ops._common import mark_shadow_fresh  # noqa: F401 - shadows re-derive from _version
    return rep


def checkpoint_keys(path: str) -> List[str]:
    return list(native().fdl_keys(path))


def checkpoint_version(path: str) -> int:
    return int(native().fdl_version(path))


def migrate_checkpoint(path_in: str, path_out: str, renames: Dict[str, str]) -> MigrateReport:
    """Rewrite entry names (old -> new) into a current-version file."""
    _, h, entries = native().read_fdl(path_in)
    rep = MigrateReport()
    out = []
    for n, t in entries:
        if n in renames:
            rep.renamed.append((n, renames[n]))
            out.append((renames[n], t))
        else:
            rep.unchanged.append(n)
            out.append((n, t))
    native().write_fdl(path_out, out, h if any(c != "0" for c in h) else None)
    return rep


migrate_checkpoint_file = migrate_checkpoint
