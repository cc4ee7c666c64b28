"""DeBERTa-v2 / v3 encoder with disentangled attention and task heads.

Reference: flodl-hf/src/models/deberta_v2.rs and deberta_transformer_layer.rs.
Attribute names follow HuggingFace's, with query/key/value packed into one
``attention.self.qkv`` Linear (see :func:`flodl_b200.models.encoders.pack_qkv`).

Attention score of query i and key j (He et al. 2021, "DeBERTa: decoding-
enhanced BERT with disentangled attention", eq. 2-4):

    ( q_i.k_j  +  q_i.Kr[d(i,j)]  +  k_j.Qr[d(i,j)] ) / sqrt(D * f)

content-to-content, content-to-position (``c2p``) and position-to-content
(``p2c``); ``Kr`` / ``Qr`` project the shared relative-position embedding
table (through the content projections when ``share_att_key``), f counts the
enabled terms, and d(i,j) = clamp(bucket(i - j) + span, 0, 2 span - 1) with
log buckets beyond ``position_buckets / 2``:
bucket(r) = r for |r| <= mid, else sign(r) (ceil(log(|r|/mid) /
log((max_rel - 1)/mid) (mid - 1)) + mid). The padding mask is pairwise
(query and key both real). The relative terms make this attention a
composed computation (batched GEMMs, gathers, masked softmax) rather than
the flash kernel.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import torch
import torch.nn.functional as F

from .. import ops
from ..nn.layers import Embedding, LayerNorm, Linear
from ..nn.module import Module
from .encoders import _act


@dataclass
class DebertaV2Config:
    vocab_size: int = 128100
    hidden_size: int = 1536
    num_hidden_layers: int = 24
    num_attention_heads: int = 24
    intermediate_size: int = 6144
    hidden_act: str = "gelu"
    max_position_embeddings: int = 512
    type_vocab_size: int = 0
    layer_norm_eps: float = 1e-7
    relative_attention: bool = False
    max_relative_positions: int = -1
    pad_token_id: int = 0
    position_biased_input: bool = True
    pos_att_type: Optional[List[str]] = None
    pooler_hidden_act: str = "gelu"
    pooler_hidden_size: Optional[int] = None
    embedding_size: Optional[int] = None
    position_buckets: int = -1
    share_att_key: bool = False
    norm_rel_ebd: str = "none"
    conv_kernel_size: int = 0
    conv_groups: int = 1
    conv_act: str = "tanh"
    legacy: bool = True
    num_labels: int = 2

    def __post_init__(self):
        if isinstance(self.pos_att_type, str):
            self.pos_att_type = [x.strip() for x in self.pos_att_type.lower().split("|")]
        self.pos_att_type = list(self.pos_att_type or [])
        if self.pooler_hidden_size is None:
            self.pooler_hidden_size = self.hidden_size
        if self.embedding_size is None:
            self.embedding_size = self.hidden_size

    @classmethod
    def from_dict(cls, d: dict) -> "DebertaV2Config":
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})

    @property
    def max_rel(self) -> int:
        return self.max_relative_positions if self.max_relative_positions >= 1 else self.max_position_embeddings

    @property
    def span(self) -> int:
        return self.position_buckets if self.position_buckets > 0 else self.max_rel


def log_bucket(rel: torch.Tensor, bucket_size: int, max_position: int) -> torch.Tensor:
    mid = bucket_size // 2
    a = rel.abs().float()
    denom = torch.log(torch.tensor((max_position - 1) / mid, device=rel.device))
    logp = torch.ceil(torch.log(a.clamp(min=1) / mid) / denom * (mid - 1)) + mid
    return torch.where(a <= mid, rel.float(), logp * torch.sign(rel.float())).long()


def relative_positions(S: int, cfg: DebertaV2Config, device) -> torch.Tensor:
    i = torch.arange(S, device=device)
    rel = i[:, None] - i[None, :]
    if cfg.position_buckets > 0 and cfg.max_rel > 0:
        rel = log_bucket(rel, cfg.position_buckets, cfg.max_rel)
    return rel


class DebertaV2Embeddings(Module):
    NAME = "deberta_embeddings"

    def __init__(self, cfg: DebertaV2Config, device=None):
        super().__init__()
        E, H = cfg.embedding_size, cfg.hidden_size
        self.word_embeddings = Embedding(cfg.vocab_size, E, device=device)
        self.position_embeddings = (Embedding(cfg.max_position_embeddings, E, device=device)
                                    if cfg.position_biased_input else None)
        self.token_type_embeddings = (Embedding(cfg.type_vocab_size, E, device=device)
                                      if cfg.type_vocab_size > 0 else None)
        self.embed_proj = Linear(E, H, bias=False, device=device) if E != H else None
        self.LayerNorm = LayerNorm(H, cfg.layer_norm_eps, device=device)

    def forward(self, ids, token_type_ids=None, mask=None):
        x = self.word_embeddings(ids)
        if self.position_embeddings is not None:
            x = x + self.position_embeddings(torch.arange(ids.shape[1], device=ids.device))[None]
        if self.token_type_embeddings is not None:
            tt = token_type_ids if token_type_ids is not None else torch.zeros_like(ids)
            x = x + self.token_type_embeddings(tt)
        if self.embed_proj is not None:
            x = self.embed_proj(x)
        x = self.LayerNorm(x)
        return x * mask[..., None].to(x.dtype) if mask is not None else x


class DisentangledSelfAttention(Module):
    NAME = "deberta_self_attention"

    def __init__(self, cfg: DebertaV2Config, device=None):
        super().__init__()
        self.cfg = cfg
        H = cfg.hidden_size
        self.heads = cfg.num_attention_heads
        self.qkv = Linear(H, 3 * H, device=device)
        self.pos_key_proj = (Linear(H, H, device=device) if cfg.relative_attention and
                             not cfg.share_att_key and "c2p" in cfg.pos_att_type else None)
        self.pos_query_proj = (Linear(H, H, device=device) if cfg.relative_attention and
                               not cfg.share_att_key and "p2c" in cfg.pos_att_type else None)

    def _heads(self, x):  # [B, S, H*D] -> [B, H, S, D]
        B, S, _ = x.shape
        return x.view(B, S, self.heads, -1).transpose(1, 2)

    def forward(self, x, pair_mask, rel_pos=None, rel_emb=None):
        cfg = self.cfg
        B, S, C = x.shape
        q, k, v = self.qkv(x).float().chunk(3, -1)
        q, k, v = self._heads(q), self._heads(k), self._heads(v)
        D = q.shape[-1]
        f = 1 + ("c2p" in cfg.pos_att_type) + ("p2c" in cfg.pos_att_type)
        scale = math.sqrt(D * f)
        scores = q @ k.transpose(-1, -2) / scale
        if cfg.relative_attention and rel_emb is not None:
            span = cfg.span
            r = rel_emb[: 2 * span].float()
            Wq, Wk, _ = self.qkv.weight.float().chunk(3, 0)
            bq, bk, _ = self.qkv.bias.float().chunk(3, 0)
            idx = torch.clamp(rel_pos + span, 0, 2 * span - 1)          # [S, S]
            if "c2p" in cfg.pos_att_type:
                pk = (F.linear(r, Wk, bk) if cfg.share_att_key
                      else self.pos_key_proj(r).float())                # [2span, C]
                pk = pk.view(2 * span, self.heads, D).transpose(0, 1)     # [H, 2span, D]
                c2p = q @ pk.transpose(-1, -2)[None]                      # [B, H, S, 2span]
                scores = scores + torch.gather(c2p, -1, idx.expand(B, self.heads, S, S)) / scale
            if "p2c" in cfg.pos_att_type:
                pq = (F.linear(r, Wq, bq) if cfg.share_att_key
                      else self.pos_query_proj(r).float())
                pq = pq.view(2 * span, self.heads, D).transpose(0, 1)
                p2c = k @ pq.transpose(-1, -2)[None]                      # [B, H, S(key), 2span]
                pidx = torch.clamp(-rel_pos + span, 0, 2 * span - 1)
                p2c = torch.gather(p2c, -1, pidx.expand(B, self.heads, S, S)).transpose(-1, -2)
                scores = scores + p2c / scale
        scores = scores.masked_fill(~pair_mask[:, None], torch.finfo(scores.dtype).min)
        o = torch.softmax(scores, -1) @ v
        return o.transpose(1, 2).reshape(B, S, C).to(x.dtype)


class _DenseLN(Module):
    NAME = "deberta_output"

    def __init__(self, din, dout, eps, device=None):
        super().__init__()
        self.dense = Linear(din, dout, device=device)
        self.LayerNorm = LayerNorm(dout, eps, device=device)

    def forward(self, h, residual):
        return self.LayerNorm(self.dense(h).to(residual.dtype) + residual)


class DebertaV2Attention(Module):
    NAME = "deberta_attention"

    def __init__(self, cfg, device=None):
        super().__init__()
        self.self = DisentangledSelfAttention(cfg, device)
        self.output = _DenseLN(cfg.hidden_size, cfg.hidden_size, cfg.layer_norm_eps, device)

    def forward(self, x, pair_mask, rel_pos, rel_emb):
        return self.output(self.self(x, pair_mask, rel_pos, rel_emb), x)


class _Intermediate(Module):
    NAME = "deberta_intermediate"

    def __init__(self, cfg, device=None):
        super().__init__()
        self.act = cfg.hidden_act
        self.dense = Linear(cfg.hidden_size, cfg.intermediate_size, device=device)

    def forward(self, x):
        return _act(self.act, self.dense(x))


class DebertaV2Layer(Module):
    NAME = "deberta_layer"

    def __init__(self, cfg, device=None):
        super().__init__()
        self.attention = DebertaV2Attention(cfg, device)
        self.intermediate = _Intermediate(cfg, device)
        self.output = _DenseLN(cfg.intermediate_size, cfg.hidden_size, cfg.layer_norm_eps, device)

    def forward(self, x, pair_mask, rel_pos, rel_emb):
        a = self.attention(x, pair_mask, rel_pos, rel_emb)
        return self.output(self.intermediate(a), a)


class _ConvLayer(Module):
    NAME = "deberta_conv"

    def __init__(self, cfg, device=None):
        super().__init__()
        k = cfg.conv_kernel_size
        self.act = cfg.conv_act
        self.conv = torch.nn.Conv1d(cfg.hidden_size, cfg.hidden_size, k, padding=(k - 1) // 2,
                                    groups=cfg.conv_groups, device=device)
        self.LayerNorm = LayerNorm(cfg.hidden_size, cfg.layer_norm_eps, device=device)

    def forward(self, h, residual, mask):
        out = self.conv(h.transpose(1, 2).float()).transpose(1, 2)
        out = out.masked_fill(~mask.bool()[..., None], 0.0)
        out = torch.tanh(out) if self.act == "tanh" else _act(self.act, out)
        return self.LayerNorm(residual + out.to(residual.dtype)) * mask[..., None].to(residual.dtype)


class DebertaV2Encoder(Module):
    NAME = "deberta_encoder"

    def __init__(self, cfg: DebertaV2Config, device=None):
        super().__init__()
        self.cfg = cfg
        self.layer = torch.nn.ModuleList([DebertaV2Layer(cfg, device) for _ in range(cfg.num_hidden_layers)])
        self.rel_embeddings = (Embedding(2 * cfg.span, cfg.hidden_size, device=device)
                               if cfg.relative_attention else None)
        norms = [x.strip() for x in cfg.norm_rel_ebd.lower().split("|")]
        self.LayerNorm = (LayerNorm(cfg.hidden_size, cfg.layer_norm_eps, device=device)
                          if "layer_norm" in norms else None)
        self.conv = _ConvLayer(cfg, device) if cfg.conv_kernel_size > 0 else None

    def forward(self, x, mask):
        m = mask.bool()
        pair = m[:, :, None] & m[:, None, :]
        rel_pos = rel_emb = None
        if self.rel_embeddings is not None:
            rel_pos = relative_positions(x.shape[1], self.cfg, x.device)
            rel_emb = self.rel_embeddings.weight
            if self.LayerNorm is not None:
                rel_emb = self.LayerNorm(rel_emb)
        h0, out = x, x
        for i, l in enumerate(self.layer):
            out = l(out, pair, rel_pos, rel_emb)
            if i == 0 and self.conv is not None:
                out = self.conv(h0, out, mask)
        return out


class DebertaV2Model(Module):
    NAME = "deberta"

    def __init__(self, cfg: DebertaV2Config, device=None):
        super().__init__()
        self.config = cfg
        self.embeddings = DebertaV2Embeddings(cfg, device)
        self.encoder = DebertaV2Encoder(cfg, device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        mask = attention_mask if attention_mask is not None else torch.ones_like(ids)
        return self.encoder(self.embeddings(ids, token_type_ids, mask), mask)


class _LegacyTransform(Module):
    NAME = "deberta_lm_transform"

    def __init__(self, cfg, device=None):
        super().__init__()
        self.act = cfg.hidden_act
        self.dense = Linear(cfg.hidden_size, cfg.embedding_size, device=device)
        self.LayerNorm = LayerNorm(cfg.embedding_size, cfg.layer_norm_eps, device=device)

    def forward(self, h):
        return self.LayerNorm(_act(self.act, self.dense(h)))


class _LegacyPredictions(Module):
    NAME = "deberta_lm_predictions"

    def __init__(self, cfg, word_embeddings, device=None):
        super().__init__()
        self.transform = _LegacyTransform(cfg, device)
        self.bias = torch.nn.Parameter(torch.zeros(cfg.vocab_size, device=device))
        self._decoder = [word_embeddings]

    def forward(self, h):
        return ops.linear(self.transform(h), self._decoder[0].weight, self.bias)


class _LegacyCls(Module):
    NAME = "deberta_cls"

    def __init__(self, cfg, word_embeddings, device=None):
        super().__init__()
        self.predictions = _LegacyPredictions(cfg, word_embeddings, device)

    def forward(self, h):
        return self.predictions(h)


class _LmHead(Module):
    NAME = "deberta_lm_head"

    def __init__(self, cfg, device=None):
        super().__init__()
        self.act = cfg.hidden_act
        self.dense = Linear(cfg.hidden_size, cfg.hidden_size, device=device)
        self.LayerNorm = LayerNorm(cfg.hidden_size, cfg.layer_norm_eps, device=device)
        self.bias = torch.nn.Parameter(torch.zeros(cfg.vocab_size, device=device))


class _LmPredictions(Module):
    NAME = "deberta_lm_preds"

    def __init__(self, cfg, device=None):
        super().__init__()
        self.lm_head = _LmHead(cfg, device)


class DebertaV2ForMaskedLM(Module):
    NAME = "deberta_mlm"

    def __init__(self, cfg: DebertaV2Config, device=None):
        super().__init__()
        self.config = cfg
        self.deberta = DebertaV2Model(cfg, device)
        if cfg.legacy:
            self.cls = _LegacyCls(cfg, self.deberta.embeddings.word_embeddings, device)
        else:
            self.lm_predictions = _LmPredictions(cfg, device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        h = self.deberta(ids, token_type_ids, attention_mask)
        if self.config.legacy:
            return self.cls(h)
        hd = self.lm_predictions.lm_head
        t = hd.LayerNorm(_act(hd.act, hd.dense(h)))
        return ops.linear(t, self.deberta.embeddings.word_embeddings.weight, hd.bias)


class ContextPooler(Module):
    NAME = "deberta_pooler"

    def __init__(self, cfg, device=None):
        super().__init__()
        self.act = cfg.pooler_hidden_act
        self.dense = Linear(cfg.pooler_hidden_size, cfg.pooler_hidden_size, device=device)

    def forward(self, h):
        return _act(self.act, self.dense(h[:, 0]))


class DebertaV2ForSequenceClassification(Module):
    NAME = "deberta_seq_cls"

    def __init__(self, cfg: DebertaV2Config, device=None):
        super().__init__()
        self.config = cfg
        self.deberta = DebertaV2Model(cfg, device)
        self.pooler = ContextPooler(cfg, device)
        self.classifier = Linear(cfg.hidden_size, cfg.num_labels, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.classifier(self.pooler(self.deberta(ids, token_type_ids, attention_mask)))


class DebertaV2ForTokenClassification(Module):
    NAME = "deberta_token_cls"

    def __init__(self, cfg: DebertaV2Config, device=None):
        super().__init__()
        self.config = cfg
        self.deberta = DebertaV2Model(cfg, device)
        self.classifier = Linear(cfg.hidden_size, cfg.num_labels, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        return self.classifier(self.deberta(ids, token_type_ids, attention_mask))


class DebertaV2ForQuestionAnswering(Module):
    NAME = "deberta_qa"

    def __init__(self, cfg: DebertaV2Config, device=None):
        super().__init__()
        self.config = cfg
        self.deberta = DebertaV2Model(cfg, device)
        self.qa_outputs = Linear(cfg.hidden_size, 2, device=device)

    def forward(self, ids, token_type_ids=None, attention_mask=None):
        s, e = self.qa_outputs(self.deberta(ids, token_type_ids, attention_mask)).split(1, -1)
        return s.squeeze(-1), e.squeeze(-1)
