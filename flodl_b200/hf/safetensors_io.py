"""safetensors reading/writing and HuggingFace checkpoint mapping
(flodl-hf/src/safetensors_io.rs:236-617).

Format: u64 little-endian header length N | N bytes of JSON
``{name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}}``
| raw little-endian tensor bytes. Files are memory-mapped for reading.
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from typing import Dict, Iterable, List, Optional, Tuple

import torch

_DT = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16, "F64": torch.float64,
       "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8,
       "U8": torch.uint8, "BOOL": torch.bool}
_DT_NAME = {v: k for k, v in _DT.items()}


def load_safetensors(path: str, device="cpu") -> Dict[str, torch.Tensor]:
    with open(path, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    try:
        (n,) = struct.unpack("<Q", mm[:8])
        if n > len(mm) - 8:
            raise ValueError(f"{path}: header length {n} exceeds file size")
        header = json.loads(mm[8:8 + n].decode("utf-8"))
        base = 8 + n
        out = {}
        for name, info in header.items():
            if name == "__metadata__":
                continue
            dt = _DT[info["dtype"]]
            b, e = info["data_offsets"]
            shape = info["shape"]
            raw = bytearray(mm[base + b:base + e])
            t = torch.frombuffer(raw, dtype=dt) if raw else torch.empty(0, dtype=dt)
            out[name] = t.reshape(shape).to(device)
        return out
    finally:
        mm.close()


def save_safetensors(path: str, tensors: Dict[str, torch.Tensor],
                     metadata: Optional[Dict[str, str]] = None) -> None:
    header = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().cpu().contiguous()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _DT_NAME[t.dtype], "shape": list(t.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


# ---------------------------------------------------------------- HF <-> flodl_b200 names
def hf_bert_to_flodl(sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Map HuggingFace BERT keys onto this package's BERT module keys (packs
    query/key/value into one qkv Linear; renames the MLM head)."""
    out: Dict[str, torch.Tensor] = {}
    qkv: Dict[str, Dict[str, torch.Tensor]] = {}
    for k, v in sd.items():
        if ".attention.self." in k:
            prefix, rest = k.split(".attention.self.")
            which, kind = rest.split(".")  # query.weight
            qkv.setdefault(f"{prefix}.attention.self.qkv.{kind}", {})[which] = v
            continue
        k2 = k
        k2 = k2.replace("cls.predictions.transform.dense.", "cls.transform_dense.")
        k2 = k2.replace("cls.predictions.transform.LayerNorm.", "cls.transform_LayerNorm.")
        k2 = k2.replace("cls.predictions.bias", "cls.bias")
        if k2.startswith("cls.predictions.decoder."):
            continue  # tied to the word embeddings
        k2 = k2.replace(".gamma", ".weight").replace(".beta", ".bias")
        out[k2] = v
    for k, parts in qkv.items():
        out[k] = torch.cat([parts["query"], parts["key"], parts["value"]], dim=0)
    return out


def flodl_bert_to_hf(sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    out: Dict[str, torch.Tensor] = {}
    for k, v in sd.items():
        if ".attention.self.qkv." in k:
            prefix, kind = k.split(".attention.self.qkv.")
            q, kk, vv = v.chunk(3, dim=0)
            for which, t in (("query", q), ("key", kk), ("value", vv)):
                out[f"{prefix}.attention.self.{which}.{kind}"] = t.contiguous()
            continue
        k2 = k.replace("cls.transform_dense.", "cls.predictions.transform.dense.")
        k2 = k2.replace("cls.transform_LayerNorm.", "cls.predictions.transform.LayerNorm.")
        k2 = k2.replace("cls.bias", "cls.predictions.bias")
        out[k2] = v
    return out


def load_into(model: torch.nn.Module, sd: Dict[str, torch.Tensor], strict: bool = True,
              prefix_candidates: Iterable[str] = ("", "bert.")) -> Tuple[List[str], List[str]]:
    """Copy tensors into ``model`` by name; returns (missing, unexpected).
    Shape mismatches raise. HF models saved without the ``bert.`` prefix are
    matched by trying the candidate prefixes."""
    own = dict(model.named_parameters())
    own.update(dict(model.named_buffers()))
    used = set()
    missing = []
    with torch.no_grad():
        for name, t in own.items():
            src = None
            for pre in prefix_candidates:
                cand = name[len(pre):] if pre and name.startswith(pre) else None
                for key in (name, cand):
                    if key is not None and key in sd:
                        src = key
                        break
                if src:
                    break
            if src is None:
                missing.append(name)
                continue
            v = sd[src]
            if tuple(v.shape) != tuple(t.shape):
                raise ValueError(f"{name}: shape mismatch: checkpoint={list(v.shape)} model={list(t.shape)}")
            t.copy_(v.to(dtype=t.dtype, device=t.device))
            used.add(src)
    unexpected = [k for k in sd if k not in used]
    if strict and missing:
        raise ValueError(f"missing keys: {missing[:8]}{'...' if len(missing) > 8 else ''}")
    return missing, unexpected
