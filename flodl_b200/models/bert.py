"""BERT family encoders (post-LayerNorm) with HuggingFace-compatible weights.

Reference: flodl-hf/src/models/bert.rs (``BertConfig::bert_base_uncased``
flodl-hf/src/models/bert.rs:102) and task heads (task_heads.rs). Parameters
use HuggingFace's names except that each layer's query/key/value projections
are packed into one ``attention.self.qkv`` Linear [3C, C] so the projection
is one tcgen05 GEMM and flash attention reads Q/K/V from its output;
:mod:`flodl_b200.hf` maps HF checkpoints (separate query/key/value) onto it.

``BertForMaskedLM.loss(ids, labels, token_type_ids, attention_mask)`` on CUDA
runs the fused post-LN training op (:mod:`flodl_b200.ops.bert`); elsewhere it
composes the modules.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from .. import ops
from ..nn.layers import Embedding, LayerNorm, Linear
from ..nn.module import Module


@dataclass
class BertConfig:
    vocab_size: int = 30522
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    max_position_embeddings: int = 512
    type_vocab_size: int = 2
    layer_norm_eps: float = 1e-12
    hidden_act: str = "gelu"
    num_labels: int = 2

    @classmethod
    def bert_base_uncased(cls) -> "BertConfig":
        return cls()

    @classmethod
    def from_dict(cls, d: dict) -> "BertConfig":
        keys = cls.__dataclass_fields__.keys()
        return cls(**{k: v for k, v in d.items() if k in keys})


class BertEmbeddings(Module):
    NAME = "bert_embeddings"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.word_embeddings = Embedding(cfg.vocab_size, cfg.hidden_size, device=device)
        self.position_embeddings = Embedding(cfg.max_position_embeddings, cfg.hidden_size, device=device)
        self.token_type_embeddings = Embedding(cfg.type_vocab_size, cfg.hidden_size, device=device)
        with torch.no_grad():
            for e in (self.word_embeddings, self.position_embeddings, self.token_type_embeddings):
                e.weight.normal_(0.0, 0.02)
        self.LayerNorm = LayerNorm(cfg.hidden_size, cfg.layer_norm_eps, device=device)

    def forward(self, ids, token_type_ids=None):
        B, S = ids.shape
        pos = torch.arange(S, device=ids.device)
        x = self.word_embeddings(ids) + self.position_embeddings(pos)[None]
        tt = token_type_ids if token_type_ids is not None else torch.zeros_like(ids)
        x = x + self.token_type_embeddings(tt)
        return self.LayerNorm(x)


class BertSelfAttention(Module):
    NAME = "bert_self_attention"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.num_heads = cfg.num_attention_heads
        self.qkv = Linear(cfg.hidden_size, 3 * cfg.hidden_size, device=device)


class BertAttention(Module):
    NAME = "bert_attention"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.self = BertSelfAttention(cfg, device)
        self.output = _DenseLN(cfg.hidden_size, cfg.hidden_size, cfg.layer_norm_eps, device)

    def forward(self, x, key_padding=None):
        B, S, C = x.shape
        qkv = self.self.qkv(x.reshape(B * S, C))
        a = ops.attention_packed(qkv, B, S, self.self.num_heads, False, key_padding)
        return self.output(a.reshape(B, S, C), x)


class _DenseLN(Module):
    """dense -> (+ residual) -> LayerNorm (BertSelfOutput / BertOutput)."""

    NAME = "bert_output"

    def __init__(self, din, dout, eps, device=None):
        super().__init__()
        self.dense = Linear(din, dout, device=device)
        self.LayerNorm = LayerNorm(dout, eps, device=device)

    def forward(self, h, residual):
        y = self.dense(h).to(residual.dtype) + residual
        return self.LayerNorm(y)


class BertIntermediate(Module):
    NAME = "bert_intermediate"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.dense = Linear(cfg.hidden_size, cfg.intermediate_size, device=device)

    def forward(self, x):
        return ops.gelu(self.dense(x))


class BertLayer(Module):
    NAME = "bert_layer"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.attention = BertAttention(cfg, device)
        self.intermediate = BertIntermediate(cfg, device)
        self.output = _DenseLN(cfg.intermediate_size, cfg.hidden_size, cfg.layer_norm_eps, device)

    def forward(self, x, key_padding=None):
        x = self.attention(x, key_padding)
        return self.output(self.intermediate(x), x)


class BertEncoder(Module):
    NAME = "bert_encoder"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.layer = torch.nn.ModuleList([BertLayer(cfg, device) for _ in range(cfg.num_hidden_layers)])

    def forward(self, x, key_padding=None):
        for l in self.layer:
            x = l(x, key_padding)
        return x


class BertPooler(Module):
    NAME = "bert_pooler"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.dense = Linear(cfg.hidden_size, cfg.hidden_size, device=device)

    def forward(self, x):
        return torch.tanh(self.dense(x[:, 0]).float())


class BertModel(Module):
    NAME = "bert"

    def __init__(self, cfg: BertConfig, add_pooler: bool = True, device=None):
        super().__init__()
        self.config = cfg
        self.embeddings = BertEmbeddings(cfg, device)
        self.encoder = BertEncoder(cfg, device)
        self.pooler = BertPooler(cfg, device) if add_pooler else None

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        key_padding = None if attention_mask is None else (attention_mask == 0)
        x = self.embeddings(ids, token_type_ids)
        return self.encoder(x, key_padding)


class BertLMPredictionHead(Module):
    NAME = "bert_lm_head"

    def __init__(self, cfg: BertConfig, word_embeddings: Embedding, device=None):
        super().__init__()
        self.transform_dense = Linear(cfg.hidden_size, cfg.hidden_size, device=device)
        self.transform_LayerNorm = LayerNorm(cfg.hidden_size, cfg.layer_norm_eps, device=device)
        self.bias = torch.nn.Parameter(torch.zeros(cfg.vocab_size, device=device))
        self._decoder = [word_embeddings]  # tied weights (not registered twice)

    @property
    def decoder_weight(self):
        return self._decoder[0].weight

    def forward(self, h):
        t = self.transform_LayerNorm(ops.gelu(self.transform_dense(h)))
        return ops.linear(t, self.decoder_weight, self.bias)


class BertForMaskedLM(Module):
    NAME = "bert_mlm"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.config = cfg
        self.bert = BertModel(cfg, add_pooler=False, device=device)
        self.cls = BertLMPredictionHead(cfg, self.bert.embeddings.word_embeddings, device)
        dev = torch.device(device) if device is not None else torch.device("cpu")
        self._grad_anchor = torch.zeros((), device=dev, requires_grad=True)

    def move_to_device(self, device):
        super().move_to_device(device)
        self._grad_anchor = torch.zeros((), device=torch.device(device), requires_grad=True)
        return self

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.cls(self.bert(ids, token_type_ids, attention_mask))

    def loss(self, ids, labels, token_type_ids=None, attention_mask=None, masked_rows=None):
        """Masked-LM loss: mean cross-entropy over positions whose label != -100.
        ``masked_rows`` (CUDA training path) fixes how many positions the head
        processes, which avoids a host sync (needed for CUDA-graph capture)."""
        if ids.is_cuda and self.training and torch.is_grad_enabled():
            return ops.bert_mlm_train_loss(self, ids, labels, token_type_ids, attention_mask,
                                           masked_rows)
        h = self.bert(ids, token_type_ids, attention_mask)
        sel = labels.reshape(-1) != -100
        hm = h.reshape(-1, h.shape[-1])[sel]
        logits = self.cls(hm)
        return ops.cross_entropy(logits, labels.reshape(-1)[sel])


class BertForSequenceClassification(Module):
    NAME = "bert_seq_cls"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.bert = BertModel(cfg, add_pooler=True, device=device)
        self.classifier = Linear(cfg.hidden_size, cfg.num_labels, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        h = self.bert(ids, token_type_ids, attention_mask)
        return self.classifier(self.bert.pooler(h))


class BertForTokenClassification(Module):
    NAME = "bert_token_cls"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.bert = BertModel(cfg, add_pooler=False, device=device)
        self.classifier = Linear(cfg.hidden_size, cfg.num_labels, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.classifier(self.bert(ids, token_type_ids, attention_mask))


class BertForQuestionAnswering(Module):
    NAME = "bert_qa"

    def __init__(self, cfg: BertConfig, device=None):
        super().__init__()
        self.bert = BertModel(cfg, add_pooler=False, device=device)
        self.qa_outputs = Linear(cfg.hidden_size, 2, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        logits = self.qa_outputs(self.bert(ids, token_type_ids, attention_mask))
        start, end = logits.split(1, dim=-1)
        return start.squeeze(-1), end.squeeze(-1)
