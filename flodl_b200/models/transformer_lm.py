"""Decoder-only transformer language model (pre-LayerNorm, GELU MLP).

The flagship DDP benchmark model: 6 layers, d_model 512, 8 heads, MLP 2048,
vocab 256 (bytes), seq 256. Reference shape: benchmarks/src/tier1/transformer.rs
(4 x 512, 8 heads, FFN 2048) and ddp-bench/src/models/gpt-nano.

Two execution paths over the same parameters:
* ``forward(ids)`` composes the framework's modules (works on CPU and CUDA).
* ``loss(ids, targets)`` on CUDA runs the fused whole-model training op
  (:mod:`flodl_b200.ops.transformer`); on CPU it composes the modules.
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..nn.layers import Embedding, LayerNorm, Linear
from ..nn.module import Module


class DecoderBlock(Module):
    NAME = "decoder_block"

    def __init__(self, d_model: int, n_heads: int, d_ff: int, causal: bool = True, device=None):
        super().__init__()
        self.n_heads = n_heads
        self.causal = causal
        self.ln1 = LayerNorm(d_model, device=device)
        self.qkv = Linear(d_model, 3 * d_model, device=device)
        self.proj = Linear(d_model, d_model, device=device)
        self.ln2 = LayerNorm(d_model, device=device)
        self.fc1 = Linear(d_model, d_ff, device=device)
        self.fc2 = Linear(d_ff, d_model, device=device)

    def forward(self, x):
        B, S, Cd = x.shape
        h = self.ln1(x)
        qkv = self.qkv(h.reshape(B * S, Cd))
        a = ops.attention_packed(qkv, B, S, self.n_heads, self.causal)
        x = x + self.proj(a).reshape(B, S, Cd).to(x.dtype)
        h = self.fc1(self.ln2(x))
        h = ops.gelu(h)
        return x + self.fc2(h).to(x.dtype)


class TransformerLM(Module):
    NAME = "transformer_lm"

    def __init__(self, vocab_size: int = 256, d_model: int = 512, n_layers: int = 6,
                 n_heads: int = 8, d_ff: int = 2048, max_seq: int = 256, causal: bool = True,
                 device=None):
        super().__init__()
        self.vocab_size, self.d_model, self.num_heads = vocab_size, d_model, n_heads
        self.max_seq, self.causal = max_seq, causal
        dev = torch.device(device) if device is not None else torch.device("cpu")
        self.tok_emb = Embedding(vocab_size, d_model, device=dev)
        with torch.no_grad():
            self.tok_emb.weight.mul_(0.02)
        self.pos_emb = torch.nn.Parameter(torch.randn(max_seq, d_model, device=dev) * 0.02)
        self.blocks = torch.nn.ModuleList(
            [DecoderBlock(d_model, n_heads, d_ff, causal, device=dev) for _ in range(n_layers)])
        self.ln_f = LayerNorm(d_model, device=dev)
        self.head = Linear(d_model, vocab_size, device=dev)
        self._grad_anchor = torch.zeros((), device=dev, requires_grad=True)

    def move_to_device(self, device):
        super().move_to_device(device)
        self._grad_anchor = torch.zeros((), device=device, requires_grad=True)
        return self

    def forward(self, ids):
        B, S = ids.shape
        x = self.tok_emb(ids) + self.pos_emb[:S].unsqueeze(0)
        for b in self.blocks:
            x = b(x)
        h = self.ln_f(x)
        return self.head(h)

    def loss(self, ids, targets):
        if ids.is_cuda and self.training and torch.is_grad_enabled():
            return ops.lm_train_loss(self, ids, targets)
        logits = self.forward(ids)
        return ops.cross_entropy(logits.reshape(-1, self.vocab_size), targets.reshape(-1))

    def flops_per_token(self, seq: int) -> float:
        """Training FLOPs per token (6 N + causal attention)."""
        n = sum(p.numel() for p in self.parameters()) - self.pos_emb.numel() - self.tok_emb.weight.numel()
        attn = 6 * 2 * len(self.blocks) * seq * self.d_model * (0.5 if self.causal else 1.0)
        return 6 * n + attn
