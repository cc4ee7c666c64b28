"""``AutoModel*`` loaders for local HuggingFace model directories and export.

Reference: flodl-hf/src/models/auto.rs:225 (dispatch on ``config.json``'s
``model_type``) and export.rs. A directory holds ``config.json`` and
``model.safetensors``; no network access is used.

Families: ``bert``, ``roberta``, ``xlm-roberta``, ``distilbert``, ``albert``,
``deberta-v2`` (also DeBERTa-v3 checkpoints, which use that model type). Each
loads into this package's modules (same names as HuggingFace except the
packed ``qkv`` projection). Keys are translated per family: query/key/value
packing, head renames, tied decoder weights dropped on load and written back
on export.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import torch

from ..models import deberta as D
from ..models import encoders as E
from ..models.bert import (BertConfig, BertForMaskedLM, BertForQuestionAnswering,
                           BertForSequenceClassification, BertForTokenClassification, BertModel)
from .safetensors_io import (flodl_bert_to_hf, hf_bert_to_flodl, load_into, load_safetensors,
                             save_safetensors)


@dataclass
class Family:
    config: Callable
    classes: Dict[str, type]
    qkv: str
    prefix: str
    to_ours: Callable[[Dict[str, torch.Tensor]], Dict[str, torch.Tensor]]
    to_hf: Callable[[torch.nn.Module, Dict[str, torch.Tensor]], Dict[str, torch.Tensor]]


def _drop(sd, prefixes):
    return {k: v for k, v in sd.items() if not any(k.startswith(p) for p in prefixes)}


def _rename(sd, table):
    out = {}
    for k, v in sd.items():
        for a, b in table:
            if k == a:
                k = b
        out[k] = v
    return out


def _tied(model, sd, word_key, entries):
    """Add the tied decoder tensors HuggingFace checkpoints carry."""
    w = sd.get(word_key)
    if w is None:
        return sd
    for wk, bias_src, bk in entries:
        if bias_src in sd:
            sd[wk] = w
            if bk:
                sd[bk] = sd[bias_src]
    return sd


def _bert_to_hf(model, sd):
    sd = flodl_bert_to_hf(sd)
    return _tied(model, sd, "bert.embeddings.word_embeddings.weight",
                 [("cls.predictions.decoder.weight", "cls.predictions.bias", "cls.predictions.decoder.bias")])


def _roberta_to_ours(sd):
    return E.pack_qkv(_drop(sd, ("lm_head.decoder.",)), "bert")


def _roberta_to_hf(model, sd):
    sd = E.unpack_qkv(sd, "bert")
    return _tied(model, sd, "roberta.embeddings.word_embeddings.weight",
                 [("lm_head.decoder.weight", "lm_head.bias", "lm_head.decoder.bias")])


_DISTIL_RENAMES = [("vocab_projector.bias", "vocab_projector_bias")]


def _distil_to_ours(sd):
    sd = _drop(sd, ("vocab_projector.weight",))
    return E.pack_qkv(_rename(sd, _DISTIL_RENAMES), "distilbert")


def _distil_to_hf(model, sd):
    sd = _rename(E.unpack_qkv(sd, "distilbert"), [(b, a) for a, b in _DISTIL_RENAMES])
    return _tied(model, sd, "distilbert.embeddings.word_embeddings.weight",
                 [("vocab_projector.weight", "vocab_projector.bias", None)])


def _albert_to_ours(sd):
    return E.pack_qkv(_drop(sd, ("predictions.decoder.",)), "albert")


def _albert_to_hf(model, sd):
    sd = E.unpack_qkv(sd, "albert")
    return _tied(model, sd, "albert.embeddings.word_embeddings.weight",
                 [("predictions.decoder.weight", "predictions.bias", "predictions.decoder.bias")])


def _deberta_to_ours(sd):
    return E.pack_qkv(_drop(sd, ("cls.predictions.decoder.", "mask_predictions.")), "deberta")


def _deberta_to_hf(model, sd):
    sd = E.unpack_qkv(sd, "deberta")
    return _tied(model, sd, "deberta.embeddings.word_embeddings.weight",
                 [("cls.predictions.decoder.weight", "cls.predictions.bias", "cls.predictions.decoder.bias")])


_ROBERTA = Family(E.RobertaConfig.from_dict,
                  {"base": E.RobertaModel, "mlm": E.RobertaForMaskedLM,
                   "seq": E.RobertaForSequenceClassification, "tok": E.RobertaForTokenClassification,
                   "qa": E.RobertaForQuestionAnswering}, "bert", "roberta.", _roberta_to_ours,
                  _roberta_to_hf)

FAMILIES: Dict[str, Family] = {
    "bert": Family(BertConfig.from_dict,
                   {"base": BertModel, "mlm": BertForMaskedLM, "seq": BertForSequenceClassification,
                    "tok": BertForTokenClassification, "qa": BertForQuestionAnswering},
                   "bert", "bert.", hf_bert_to_flodl, _bert_to_hf),
    "roberta": _ROBERTA,
    "xlm-roberta": _ROBERTA,
    "distilbert": Family(E.DistilBertConfig.from_dict,
                         {"base": E.DistilBertModel, "mlm": E.DistilBertForMaskedLM,
                          "seq": E.DistilBertForSequenceClassification,
                          "tok": E.DistilBertForTokenClassification,
                          "qa": E.DistilBertForQuestionAnswering},
                         "distilbert", "distilbert.", _distil_to_ours, _distil_to_hf),
    "albert": Family(E.AlbertConfig.from_dict,
                     {"base": E.AlbertModel, "mlm": E.AlbertForMaskedLM,
                      "seq": E.AlbertForSequenceClassification, "tok": E.AlbertForTokenClassification,
                      "qa": E.AlbertForQuestionAnswering},
                     "albert", "albert.", _albert_to_ours, _albert_to_hf),
    "deberta-v2": Family(D.DebertaV2Config.from_dict,
                         {"base": D.DebertaV2Model, "mlm": D.DebertaV2ForMaskedLM,
                          "seq": D.DebertaV2ForSequenceClassification,
                          "tok": D.DebertaV2ForTokenClassification,
                          "qa": D.DebertaV2ForQuestionAnswering},
                         "deberta", "deberta.", _deberta_to_ours, _deberta_to_hf),
}
RECOGNISED = set(FAMILIES)
BERT_LIKE = {"bert", "roberta", "xlm-roberta"}


HUB_FILES = ["config.json", "model.safetensors", "tokenizer.json"]


def resolve_model_dir(name_or_path: str) -> str:
    """A local directory as is; otherwise a Hub repo id resolved through the
    HuggingFace cache (``huggingface_hub.snapshot_download``; with
    ``HF_HUB_OFFLINE=1`` only the cache is consulted)."""
    if os.path.isdir(name_or_path):
        return name_or_path
    try:
        from huggingface_hub import snapshot_download
    except ImportError as e:
        raise FileNotFoundError(f"{name_or_path!r} is not a directory and huggingface_hub is "
                                f"not installed") from e
    offline = os.environ.get("HF_HUB_OFFLINE", "0") not in ("0", "", "false", "False")
    try:
        return snapshot_download(repo_id=name_or_path, allow_patterns=HUB_FILES,
                                 local_files_only=offline)
    except Exception as e:
        raise FileNotFoundError(f"{name_or_path!r}: not a local directory and not resolvable "
                                f"from the HuggingFace Hub{' cache' if offline else ''}: {e}") from e


def _read_config(path: str) -> dict:
    with open(os.path.join(path, "config.json")) as f:
        return json.load(f)


def _family_of(model) -> Tuple[str, Family]:
    for mt, fam in FAMILIES.items():
        if type(model) in fam.classes.values():
            return mt, fam
    raise ValueError(f"{type(model).__name__} is not a HuggingFace-family model of this package")


def _align_prefix(sd: Dict[str, torch.Tensor], own: List[str], prefix: str) -> Dict[str, torch.Tensor]:
    """A base model (keys without ``prefix``) loads from a head checkpoint and
    vice versa."""
    ours_prefixed = any(k.startswith(prefix) for k in own)
    theirs_prefixed = any(k.startswith(prefix) for k in sd)
    if theirs_prefixed and not ours_prefixed:
        return {k[len(prefix):]: v for k, v in sd.items() if k.startswith(prefix)}
    if ours_prefixed and not theirs_prefixed:
        heads = {k for k in own if not k.startswith(prefix)}
        return {(k if k in heads else prefix + k): v for k, v in sd.items()}
    return sd


def _load(kind: str, path: str, device=None, strict: bool = False):
    path = resolve_model_dir(path)
    cfgd = _read_config(path)
    mt = cfgd.get("model_type", "bert")
    if mt not in RECOGNISED:
        raise ValueError(f"unsupported model_type {mt!r} (known: {sorted(RECOGNISED)})")
    if mt not in FAMILIES:
        raise NotImplementedError(f"model_type {mt!r} is recognised but has no module here yet")
    fam = FAMILIES[mt]
    cfg = fam.config(cfgd)
    if "id2label" in cfgd and "num_labels" not in cfgd:
        cfg.num_labels = len(cfgd["id2label"])
    model = fam.classes[kind](cfg, device=device)
    sd = fam.to_ours(load_safetensors(os.path.join(path, "model.safetensors")))
    own = list(dict(model.named_parameters()).keys()) + [k for k, _ in model.named_buffers()]
    sd = _align_prefix(sd, own, fam.prefix)
    missing, _ = load_into(model, sd, strict=False, prefix_candidates=("",))
    if strict and missing:
        raise ValueError(f"missing keys: {missing[:8]}")
    model.load_report = missing
    return model


class _Auto:
    KIND = "base"

    @classmethod
    def from_pretrained(cls, path: str, device=None, strict: bool = False):
        return _load(cls.KIND, path, device, strict)


class AutoModel(_Auto):
    KIND = "base"


class AutoModelForMaskedLM(_Auto):
    KIND = "mlm"


class AutoModelForSequenceClassification(_Auto):
    KIND = "seq"


class AutoModelForTokenClassification(_Auto):
    KIND = "tok"


class AutoModelForQuestionAnswering(_Auto):
    KIND = "qa"


_ARCH = {"base": "Model", "mlm": "ForMaskedLM", "seq": "ForSequenceClassification",
         "tok": "ForTokenClassification", "qa": "ForQuestionAnswering"}
_HF_NAME = {"bert": "Bert", "roberta": "Roberta", "xlm-roberta": "XLMRoberta",
            "distilbert": "DistilBert", "albert": "Albert", "deberta-v2": "DebertaV2"}


def export_hf(model, path: str, model_type: Optional[str] = None) -> None:
    """Write ``config.json`` + ``model.safetensors`` loadable by HF transformers."""
    mt, fam = _family_of(model)
    mt = model_type or mt
    kind = next(k for k, c in fam.classes.items() if c is type(model))
    os.makedirs(path, exist_ok=True)
    cfg = model.config
    d = dict(cfg.__dict__)
    d["model_type"] = mt
    d["architectures"] = [_HF_NAME.get(mt, "Bert") + _ARCH[kind]]
    if kind in ("seq", "tok"):
        d["id2label"] = {str(i): f"LABEL_{i}" for i in range(cfg.num_labels)}
        d["label2id"] = {f"LABEL_{i}": i for i in range(cfg.num_labels)}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(d, f, indent=2)
    sd = {k: v.detach().cpu().contiguous() for k, v in model.state_dict().items()}
    save_safetensors(os.path.join(path, "model.safetensors"), fam.to_hf(model, sd), {"format": "pt"})
