"""``AutoModel*`` loaders for local HuggingFace model directories
(flodl-hf/src/models/auto.rs:225). A directory holds ``config.json`` and
``model.safetensors``; no network access is used. Supported ``model_type``:
bert, roberta, distilbert, albert, xlm-roberta, deberta-v2 are recognised;
BERT-family layouts (bert, roberta, xlm-roberta) load into the BERT modules.
"""
from __future__ import annotations

import json
import os

import torch

from ..models.bert import (BertConfig, BertForMaskedLM, BertForQuestionAnswering,
                           BertForSequenceClassification, BertForTokenClassification, BertModel)
from .safetensors_io import (flodl_bert_to_hf, hf_bert_to_flodl, load_into, load_safetensors,
                             save_safetensors)

BERT_LIKE = {"bert", "roberta", "xlm-roberta"}
KNOWN = BERT_LIKE | {"distilbert", "albert", "deberta-v2"}


def _read_config(path: str) -> dict:
    with open(os.path.join(path, "config.json")) as f:
        return json.load(f)


def _load(cls, path: str, device=None, **kw):
    cfgd = _read_config(path)
    mt = cfgd.get("model_type", "bert")
    if mt not in KNOWN:
        raise ValueError(f"unsupported model_type {mt!r}")
    if mt not in BERT_LIKE:
        raise NotImplementedError(f"model_type {mt!r} is recognised but not yet loadable")
    cfg = BertConfig.from_dict(cfgd)
    model = cls(cfg, device=device, **kw) if cls is not BertModel else cls(cfg, device=device)
    sd = load_safetensors(os.path.join(path, "model.safetensors"))
    load_into(model, hf_bert_to_flodl(sd), strict=False)
    return model


class AutoModel:
    @staticmethod
    def from_pretrained(path: str, device=None):
        return _load(BertModel, path, device)


class AutoModelForMaskedLM:
    @staticmethod
    def from_pretrained(path: str, device=None):
        return _load(BertForMaskedLM, path, device)


class AutoModelForSequenceClassification:
    @staticmethod
    def from_pretrained(path: str, device=None):
        return _load(BertForSequenceClassification, path, device)


class AutoModelForTokenClassification:
    @staticmethod
    def from_pretrained(path: str, device=None):
        return _load(BertForTokenClassification, path, device)


class AutoModelForQuestionAnswering:
    @staticmethod
    def from_pretrained(path: str, device=None):
        return _load(BertForQuestionAnswering, path, device)


def export_hf(model, path: str, model_type: str = "bert") -> None:
    """Write ``config.json`` + ``model.safetensors`` loadable by HF transformers."""
    os.makedirs(path, exist_ok=True)
    cfg = model.config if hasattr(model, "config") else model.bert.config
    d = dict(cfg.__dict__)
    d["model_type"] = model_type
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(d, f, indent=2)
    sd = {k: v for k, v in model.state_dict().items()}
    save_safetensors(os.path.join(path, "model.safetensors"), flodl_bert_to_hf(sd),
                     {"format": "pt"})
