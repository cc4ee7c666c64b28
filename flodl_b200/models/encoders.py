"""RoBERTa / XLM-RoBERTa, DistilBERT and ALBERT encoders with task heads.

Reference: flodl-hf/src/models/{roberta,distilbert,albert}.rs and
task_heads.rs. Module attribute names follow HuggingFace's so checkpoints map
by name, except that every attention block packs its query/key/value
projections into one ``qkv`` Linear [3C, C] (one tcgen05 GEMM feeding the flash
kernel); :func:`pack_qkv` / :func:`unpack_qkv` translate the keys.

Differences from BERT that matter for parity with HuggingFace:

* RoBERTa positions start at ``pad_token_id + 1`` and skip padding
  (``cumsum(ids != pad) * (ids != pad) + pad``); its classification head is
  ``dense -> tanh -> out_proj`` on token 0 (no pooler); the MLM head is
  ``dense -> gelu -> layer_norm -> decoder (tied) + bias``.
* DistilBERT has no token types and no pooler; layers are post-LN with
  ``sa_layer_norm`` / ``output_layer_norm``; classification is
  ``pre_classifier -> ReLU -> classifier`` on token 0.
* ALBERT factorises the embedding (E < H) with ``embedding_hidden_mapping_in``,
  shares layer weights across depth (``num_hidden_groups`` groups), uses
  ``gelu_new`` (tanh approximation), and its MLM head projects back to E.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch
import torch.nn.functional as F

from .. import ops
from ..nn.layers import Embedding, LayerNorm, Linear
from ..nn.module import Module
from .bert import BertConfig, BertEmbeddings, BertModel


def _act(name: str, x):
    if name in ("gelu_new", "gelu_pytorch_tanh", "gelu_fast"):
        return F.gelu(x.float(), approximate="tanh").to(x.dtype)
    if name == "relu":
        return F.relu(x)
    return ops.gelu(x)


def _attn(qkv_lin: Linear, x, heads: int, key_padding):
    B, S, C = x.shape
    qkv = qkv_lin(x.reshape(B * S, C))
    return ops.attention_packed(qkv, B, S, heads, False, key_padding).reshape(B, S, C)


# ----------------------------------------------------------------- key packing
QKV_PATTERNS = {
    "bert": (".attention.self.query.", ".attention.self.key.", ".attention.self.value.",
             ".attention.self.qkv."),
    "distilbert": (".attention.q_lin.", ".attention.k_lin.", ".attention.v_lin.", ".attention.qkv."),
    "albert": (".attention.query.", ".attention.key.", ".attention.value.", ".attention.qkv."),
    "deberta": (".attention.self.query_proj.", ".attention.self.key_proj.",
                ".attention.self.value_proj.", ".attention.self.qkv."),
}


def pack_qkv(sd: Dict[str, torch.Tensor], family: str) -> Dict[str, torch.Tensor]:
    q, k, v, packed = QKV_PATTERNS[family]
    out, parts = {}, {}
    for name, t in sd.items():
        for i, pat in enumerate((q, k, v)):
            if pat in name:
                parts.setdefault(name.replace(pat, packed), [None] * 3)[i] = t
                break
        else:
            out[name] = t
    for name, (tq, tk, tv) in parts.items():
        if tq is None or tk is None or tv is None:
            raise ValueError(f"incomplete query/key/value set for {name}")
        out[name] = torch.cat([tq, tk, tv], 0)
    return out


def unpack_qkv(sd: Dict[str, torch.Tensor], family: str) -> Dict[str, torch.Tensor]:
    q, k, v, packed = QKV_PATTERNS[family]
    out = {}
    for name, t in sd.items():
        if packed in name:
            for pat, part in zip((q, k, v), t.chunk(3, 0)):
                out[name.replace(packed, pat)] = part.contiguous()
        else:
            out[name] = t
    return out


# ----------------------------------------------------------------- RoBERTa / XLM-R
@dataclass
class RobertaConfig(BertConfig):
    vocab_size: int = 50265
    max_position_embeddings: int = 514
    type_vocab_size: int = 1
    layer_norm_eps: float = 1e-5
    pad_token_id: int = 1

    @classmethod
    def roberta_base(cls) -> "RobertaConfig":
        return cls()

    @classmethod
    def xlm_roberta_base(cls) -> "RobertaConfig":
        return cls(vocab_size=250002)


class RobertaEmbeddings(BertEmbeddings):
    NAME = "roberta_embeddings"

    def __init__(self, cfg: RobertaConfig, device=None):
        super().__init__(cfg, device)
        self.pad = cfg.pad_token_id

    def forward(self, ids, token_type_ids=None):
        m = (ids != self.pad).long()
        pos = torch.cumsum(m, 1) * m + self.pad
        x = self.word_embeddings(ids) + self.position_embeddings(pos)
        tt = token_type_ids if token_type_ids is not None else torch.zeros_like(ids)
        return self.LayerNorm(x + self.token_type_embeddings(tt))


class RobertaModel(BertModel):
    NAME = "roberta"

    def __init__(self, cfg: RobertaConfig, add_pooler: bool = False, device=None):
        super().__init__(cfg, add_pooler, device)
        self.embeddings = RobertaEmbeddings(cfg, device)


class RobertaLMHead(Module):
    NAME = "roberta_lm_head"

    def __init__(self, cfg: RobertaConfig, word_embeddings: Embedding, device=None):
        super().__init__()
        self.dense = Linear(cfg.hidden_size, cfg.hidden_size, device=device)
        self.layer_norm = LayerNorm(cfg.hidden_size, cfg.layer_norm_eps, device=device)
        self.bias = torch.nn.Parameter(torch.zeros(cfg.vocab_size, device=device))
        self._decoder = [word_embeddings]

    def forward(self, h):
        t = self.layer_norm(ops.gelu(self.dense(h)))
        return ops.linear(t, self._decoder[0].weight, self.bias)


class RobertaForMaskedLM(Module):
    NAME = "roberta_mlm"

    def __init__(self, cfg: RobertaConfig, device=None):
        super().__init__()
        self.config = cfg
        self.roberta = RobertaModel(cfg, device=device)
        self.lm_head = RobertaLMHead(cfg, self.roberta.embeddings.word_embeddings, device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.lm_head(self.roberta(ids, token_type_ids, attention_mask))


class RobertaClassificationHead(Module):
    NAME = "roberta_cls_head"

    def __init__(self, cfg: RobertaConfig, device=None):
        super().__init__()
        self.dense = Linear(cfg.hidden_size, cfg.hidden_size, device=device)
        self.out_proj = Linear(cfg.hidden_size, cfg.num_labels, device=device)

    def forward(self, h):
        return self.out_proj(torch.tanh(self.dense(h[:, 0]).float()))


class RobertaForSequenceClassification(Module):
    NAME = "roberta_seq_cls"

    def __init__(self, cfg: RobertaConfig, device=None):
        super().__init__()
        self.config = cfg
        self.roberta = RobertaModel(cfg, device=device)
        self.classifier = RobertaClassificationHead(cfg, device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.classifier(self.roberta(ids, token_type_ids, attention_mask))


class RobertaForTokenClassification(Module):
    NAME = "roberta_token_cls"

    def __init__(self, cfg: RobertaConfig, device=None):
        super().__init__()
        self.config = cfg
        self.roberta = RobertaModel(cfg, device=device)
        self.classifier = Linear(cfg.hidden_size, cfg.num_labels, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.classifier(self.roberta(ids, token_type_ids, attention_mask))


class RobertaForQuestionAnswering(Module):
    NAME = "roberta_qa"

    def __init__(self, cfg: RobertaConfig, device=None):
        super().__init__()
        self.config = cfg
        self.roberta = RobertaModel(cfg, device=device)
        self.qa_outputs = Linear(cfg.hidden_size, 2, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        s, e = self.qa_outputs(self.roberta(ids, token_type_ids, attention_mask)).split(1, -1)
        return s.squeeze(-1), e.squeeze(-1)


# ----------------------------------------------------------------- DistilBERT
@dataclass
class DistilBertConfig:
    vocab_size: int = 30522
    dim: int = 768
    n_layers: int = 6
    n_heads: int = 12
    hidden_dim: int = 3072
    max_position_embeddings: int = 512
    activation: str = "gelu"
    num_labels: int = 2
    layer_norm_eps: float = 1e-12

    @classmethod
    def from_dict(cls, d: dict) -> "DistilBertConfig":
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})


class DistilBertEmbeddings(Module):
    NAME = "distilbert_embeddings"

    def __init__(self, cfg: DistilBertConfig, device=None):
        super().__init__()
        self.word_embeddings = Embedding(cfg.vocab_size, cfg.dim, device=device)
        self.position_embeddings = Embedding(cfg.max_position_embeddings, cfg.dim, device=device)
        self.LayerNorm = LayerNorm(cfg.dim, cfg.layer_norm_eps, device=device)

    def forward(self, ids):
        pos = torch.arange(ids.shape[1], device=ids.device)
        return self.LayerNorm(self.word_embeddings(ids) + self.position_embeddings(pos)[None])


class _DistilAttention(Module):
    NAME = "distilbert_attention"

    def __init__(self, cfg: DistilBertConfig, device=None):
        super().__init__()
        self.heads = cfg.n_heads
        self.qkv = Linear(cfg.dim, 3 * cfg.dim, device=device)
        self.out_lin = Linear(cfg.dim, cfg.dim, device=device)

    def forward(self, x, key_padding):
        return self.out_lin(_attn(self.qkv, x, self.heads, key_padding))


class _DistilFFN(Module):
    NAME = "distilbert_ffn"

    def __init__(self, cfg: DistilBertConfig, device=None):
        super().__init__()
        self.act = cfg.activation
        self.lin1 = Linear(cfg.dim, cfg.hidden_dim, device=device)
        self.lin2 = Linear(cfg.hidden_dim, cfg.dim, device=device)

    def forward(self, x):
        return self.lin2(_act(self.act, self.lin1(x)))


class DistilBertLayer(Module):
    NAME = "distilbert_layer"

    def __init__(self, cfg: DistilBertConfig, device=None):
        super().__init__()
        self.attention = _DistilAttention(cfg, device)
        self.sa_layer_norm = LayerNorm(cfg.dim, cfg.layer_norm_eps, device=device)
        self.ffn = _DistilFFN(cfg, device)
        self.output_layer_norm = LayerNorm(cfg.dim, cfg.layer_norm_eps, device=device)

    def forward(self, x, key_padding=None):
        x = self.sa_layer_norm(self.attention(x, key_padding).to(x.dtype) + x)
        return self.output_layer_norm(self.ffn(x).to(x.dtype) + x)


class _DistilTransformer(Module):
    NAME = "distilbert_transformer"

    def __init__(self, cfg, device=None):
        super().__init__()
        self.layer = torch.nn.ModuleList([DistilBertLayer(cfg, device) for _ in range(cfg.n_layers)])

    def forward(self, x, key_padding=None):
        for l in self.layer:
            x = l(x, key_padding)
        return x


class DistilBertModel(Module):
    NAME = "distilbert"

    def __init__(self, cfg: DistilBertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.embeddings = DistilBertEmbeddings(cfg, device)
        self.transformer = _DistilTransformer(cfg, device)

    def forward(self, ids, attention_mask=None):
        kp = None if attention_mask is None else attention_mask == 0
        return self.transformer(self.embeddings(ids), kp)


class DistilBertForMaskedLM(Module):
    NAME = "distilbert_mlm"

    def __init__(self, cfg: DistilBertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.distilbert = DistilBertModel(cfg, device)
        self.vocab_transform = Linear(cfg.dim, cfg.dim, device=device)
        self.vocab_layer_norm = LayerNorm(cfg.dim, cfg.layer_norm_eps, device=device)
        self.vocab_projector_bias = torch.nn.Parameter(torch.zeros(cfg.vocab_size, device=device))

    def forward(self, ids, attention_mask=None):
        h = self.distilbert(ids, attention_mask)
        t = self.vocab_layer_norm(_act(self.config.activation, self.vocab_transform(h)))
        return ops.linear(t, self.distilbert.embeddings.word_embeddings.weight,
                          self.vocab_projector_bias)


class DistilBertForSequenceClassification(Module):
    NAME = "distilbert_seq_cls"

    def __init__(self, cfg: DistilBertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.distilbert = DistilBertModel(cfg, device)
        self.pre_classifier = Linear(cfg.dim, cfg.dim, device=device)
        self.classifier = Linear(cfg.dim, cfg.num_labels, device=device)

    def forward(self, ids, attention_mask=None):
        h = self.distilbert(ids, attention_mask)[:, 0]
        return self.classifier(F.relu(self.pre_classifier(h)))


class DistilBertForTokenClassification(Module):
    NAME = "distilbert_token_cls"

    def __init__(self, cfg: DistilBertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.distilbert = DistilBertModel(cfg, device)
        self.classifier = Linear(cfg.dim, cfg.num_labels, device=device)

    def forward(self, ids, attention_mask=None):
        return self.classifier(self.distilbert(ids, attention_mask))


class DistilBertForQuestionAnswering(Module):
    NAME = "distilbert_qa"

    def __init__(self, cfg: DistilBertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.distilbert = DistilBertModel(cfg, device)
        self.qa_outputs = Linear(cfg.dim, 2, device=device)

    def forward(self, ids, attention_mask=None):
        s, e = self.qa_outputs(self.distilbert(ids, attention_mask)).split(1, -1)
        return s.squeeze(-1), e.squeeze(-1)


# ----------------------------------------------------------------- ALBERT
@dataclass
class AlbertConfig:
    vocab_size: int = 30000
    embedding_size: int = 128
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_hidden_groups: int = 1
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    inner_group_num: int = 1
    hidden_act: str = "gelu_new"
    max_position_embeddings: int = 512
    type_vocab_size: int = 2
    layer_norm_eps: float = 1e-12
    num_labels: int = 2

    @classmethod
    def from_dict(cls, d: dict) -> "AlbertConfig":
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})


class AlbertEmbeddings(BertEmbeddings):
    NAME = "albert_embeddings"

    def __init__(self, cfg: AlbertConfig, device=None):
        bc = BertConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.embedding_size,
                        max_position_embeddings=cfg.max_position_embeddings,
                        type_vocab_size=cfg.type_vocab_size, layer_norm_eps=cfg.layer_norm_eps)
        super().__init__(bc, device)


class _AlbertAttention(Module):
    NAME = "albert_attention"

    def __init__(self, cfg: AlbertConfig, device=None):
        super().__init__()
        self.heads = cfg.num_attention_heads
        self.qkv = Linear(cfg.hidden_size, 3 * cfg.hidden_size, device=device)
        self.dense = Linear(cfg.hidden_size, cfg.hidden_size, device=device)
        self.LayerNorm = LayerNorm(cfg.hidden_size, cfg.layer_norm_eps, device=device)

    def forward(self, x, key_padding):
        return self.LayerNorm(self.dense(_attn(self.qkv, x, self.heads, key_padding)).to(x.dtype) + x)


class AlbertLayer(Module):
    NAME = "albert_layer"

    def __init__(self, cfg: AlbertConfig, device=None):
        super().__init__()
        self.act = cfg.hidden_act
        self.attention = _AlbertAttention(cfg, device)
        self.ffn = Linear(cfg.hidden_size, cfg.intermediate_size, device=device)
        self.ffn_output = Linear(cfg.intermediate_size, cfg.hidden_size, device=device)
        self.full_layer_layer_norm = LayerNorm(cfg.hidden_size, cfg.layer_norm_eps, device=device)

    def forward(self, x, key_padding=None):
        a = self.attention(x, key_padding)
        h = self.ffn_output(_act(self.act, self.ffn(a)))
        return self.full_layer_layer_norm(h.to(a.dtype) + a)


class _AlbertLayerGroup(Module):
    NAME = "albert_layer_group"

    def __init__(self, cfg, device=None):
        super().__init__()
        self.albert_layers = torch.nn.ModuleList([AlbertLayer(cfg, device)
                                                  for _ in range(cfg.inner_group_num)])

    def forward(self, x, key_padding=None):
        for l in self.albert_layers:
            x = l(x, key_padding)
        return x


class _AlbertEncoder(Module):
    NAME = "albert_encoder"

    def __init__(self, cfg: AlbertConfig, device=None):
        super().__init__()
        self.cfg = cfg
        self.embedding_hidden_mapping_in = Linear(cfg.embedding_size, cfg.hidden_size, device=device)
        self.albert_layer_groups = torch.nn.ModuleList([_AlbertLayerGroup(cfg, device)
                                                        for _ in range(cfg.num_hidden_groups)])

    def forward(self, x, key_padding=None):
        x = self.embedding_hidden_mapping_in(x)
        per = self.cfg.num_hidden_layers // self.cfg.num_hidden_groups
        for i in range(self.cfg.num_hidden_layers):  # weights shared across depth
            x = self.albert_layer_groups[i // per](x, key_padding)
        return x


class AlbertModel(Module):
    NAME = "albert"

    def __init__(self, cfg: AlbertConfig, add_pooler: bool = True, device=None):
        super().__init__()
        self.config = cfg
        self.embeddings = AlbertEmbeddings(cfg, device)
        self.encoder = _AlbertEncoder(cfg, device)
        self.pooler = Linear(cfg.hidden_size, cfg.hidden_size, device=device) if add_pooler else None

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        kp = None if attention_mask is None else attention_mask == 0
        return self.encoder(self.embeddings(ids, token_type_ids), kp)

    def pooled(self, h):
        return torch.tanh(self.pooler(h[:, 0]).float())


class AlbertForMaskedLM(Module):
    NAME = "albert_mlm"

    def __init__(self, cfg: AlbertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.albert = AlbertModel(cfg, add_pooler=False, device=device)
        self.predictions = _AlbertMLMHead(cfg, self.albert.embeddings.word_embeddings, device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.predictions(self.albert(ids, token_type_ids, attention_mask))


class _AlbertMLMHead(Module):
    NAME = "albert_mlm_head"

    def __init__(self, cfg: AlbertConfig, word_embeddings, device=None):
        super().__init__()
        self.act = cfg.hidden_act
        self.dense = Linear(cfg.hidden_size, cfg.embedding_size, device=device)
        self.LayerNorm = LayerNorm(cfg.embedding_size, cfg.layer_norm_eps, device=device)
        self.bias = torch.nn.Parameter(torch.zeros(cfg.vocab_size, device=device))
        self._decoder = [word_embeddings]

    def forward(self, h):
        t = self.LayerNorm(_act(self.act, self.dense(h)))
        return ops.linear(t, self._decoder[0].weight, self.bias)


class AlbertForSequenceClassification(Module):
    NAME = "albert_seq_cls"

    def __init__(self, cfg: AlbertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.albert = AlbertModel(cfg, device=device)
        self.classifier = Linear(cfg.hidden_size, cfg.num_labels, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.classifier(self.albert.pooled(self.albert(ids, token_type_ids, attention_mask)))


class AlbertForTokenClassification(Module):
    NAME = "albert_token_cls"

    def __init__(self, cfg: AlbertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.albert = AlbertModel(cfg, add_pooler=False, device=device)
        self.classifier = Linear(cfg.hidden_size, cfg.num_labels, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.classifier(self.albert(ids, token_type_ids, attention_mask))


class AlbertForQuestionAnswering(Module):
    NAME = "albert_qa"

    def __init__(self, cfg: AlbertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.albert = AlbertModel(cfg, add_pooler=False, device=device)
        self.qa_outputs = Linear(cfg.hidden_size, 2, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        s, e = self.qa_outputs(self.albert(ids, token_type_ids, attention_mask)).split(1, -1)
        return s.squeeze(-1), e.squeeze(-1)
