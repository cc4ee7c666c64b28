"""Model zoo of the DDP benchmark harness.

Same models, shapes, optimizers and defaults as the reference's ddp-bench zoo
(ddp-bench/src/models/*.rs): logistic regression, 2-layer MLP and LeNet-5 on
MNIST-shaped data, a convolutional autoencoder, a 2-layer LSTM char-RNN and a
GPT-nano on Shakespeare-shaped character data, ResNet-20 on CIFAR-shaped data,
and an OLMo-150M-style decoder (RMSNorm, RoPE, SwiGLU, no biases). Datasets
are synthetic with the real datasets' shapes (this machine has no network);
``flodl_b200.data.datasets`` loads the real files when they are present.

``ZOO[name]`` is a :class:`ModelDef` with ``build(device)``, ``dataset(n)``,
``train_fn(model, batch) -> loss``, ``optimizer(params, lr)`` and defaults.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict

import torch
import torch.nn.functional as F

from ..data import TensorDataSet
from ..graph import FlowBuilder
from ..nn import (LSTM, ConvTranspose2d, Conv2d, Embedding, Flatten, Linear, MaxPool2d, ReLU,
                  RMSNorm, Sigmoid)
from ..nn.module import Module
from ..optim import SGD, Adam, AdamW, RMSprop


@dataclass
class ModelDef:
    name: str
    description: str
    build: Callable
    dataset: Callable
    train_fn: Callable
    optimizer: Callable
    batch_size: int = 64
    lr: float = 1e-3
    epochs: int = 1
    extra: dict = field(default_factory=dict)


# ------------------------------------------------------------------ data (synthetic, real shapes)
def _images(n, shape, classes, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, *shape, generator=g)
    y = torch.randint(0, classes, (n,), generator=g)
    return TensorDataSet(x, y)


def _chars(n, seq, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    stream = torch.randint(0, vocab, (n * seq + 1,), generator=g)
    x = stream[:-1].view(n, seq)
    y = stream[1:].view(n, seq)
    return TensorDataSet(x, y)


def _ce(model, batch):
    x, y = batch
    return F.cross_entropy(model(x).float(), y)


def _seq_ce(model, batch):
    x, y = batch
    logits = model(x)
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), y.reshape(-1))


# ------------------------------------------------------------------ MNIST models
def _logistic(device):
    return FlowBuilder.from_(Flatten()).through(Linear(784, 10, device=device)).build()


def _mlp(device):
    return (FlowBuilder.from_(Flatten()).through(Linear(784, 256, device=device)).through(ReLU())
            .through(Linear(256, 10, device=device)).build())


def _lenet(device):
    return (FlowBuilder.from_(Conv2d(1, 6, 5, device=device)).through(ReLU()).through(MaxPool2d(2))
            .through(Conv2d(6, 16, 5, device=device)).through(ReLU()).through(MaxPool2d(2))
            .through(Flatten()).through(Linear(256, 120, device=device)).through(ReLU())
            .through(Linear(120, 84, device=device)).through(ReLU())
            .through(Linear(84, 10, device=device)).build())


def _conv_ae(device):
    return (FlowBuilder.from_(Conv2d(1, 16, 3, stride=2, padding=1, device=device)).through(ReLU())
            .through(Conv2d(16, 32, 3, stride=2, padding=1, device=device)).through(ReLU())
            .through(ConvTranspose2d(32, 16, 3, stride=2, padding=1, output_padding=1, device=device))
            .through(ReLU())
            .through(ConvTranspose2d(16, 1, 3, stride=2, padding=1, output_padding=1, device=device))
            .through(Sigmoid()).build())


def _recon(model, batch):
    x, _ = batch
    x01 = torch.sigmoid(x)
    return F.mse_loss(model(x01).float(), x01)


# ------------------------------------------------------------------ char models
class CharRNN(Module):
    """Embedding(65,128) -> LSTM(128,256, 2 layers) -> Linear(256,65) (char_rnn.rs)."""

    NAME = "char_rnn"

    def __init__(self, vocab=65, embed=128, hidden=256, layers=2, device=None):
        super().__init__()
        self.emb = Embedding(vocab, embed, device=device)
        self.lstm = LSTM(embed, hidden, layers, batch_first=True, device=device)
        self.head = Linear(hidden, vocab, device=device)

    def forward(self, ids):
        self.lstm.reset()  # each batch is an independent set of sequences
        return self.head(self.lstm(self.emb(ids)))


def _gpt_nano(device):
    from .transformer_lm import TransformerLM
    return TransformerLM(vocab_size=65, d_model=128, n_layers=4, n_heads=4, d_ff=512, max_seq=128,
                         device=device)


def _lm_loss(model, batch):
    x, y = batch
    return model.loss(x, y)


# ------------------------------------------------------------------ OLMo-style decoder
def rope_cache(seq, dim, base=10000.0, device=None):
    inv = 1.0 / (base ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    t = torch.arange(seq, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    return f.cos(), f.sin()


def apply_rope(x, cos, sin):
    """x [B, H, S, D]: rotary position embedding, half-split form - element i
    and element i + D/2 form the rotated pair, angle position * base^(-2i/D)."""
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    c, s = cos[: x.shape[-2]], sin[: x.shape[-2]]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


class OLMoBlock(Module):
    NAME = "olmo_block"

    def __init__(self, d, h, ff, device=None):
        super().__init__()
        self.h = h
        self.attn_norm = RMSNorm(d, eps=1e-6, device=device)
        self.att_proj = Linear(d, 3 * d, bias=False, device=device)
        self.attn_out = Linear(d, d, bias=False, device=device)
        self.ff_norm = RMSNorm(d, eps=1e-6, device=device)
        self.ff_proj = Linear(d, 2 * ff, bias=False, device=device)  # SwiGLU: value | gate
        self.ff_out = Linear(ff, d, bias=False, device=device)

    def forward(self, x, cos, sin):
        B, S, C = x.shape
        q, k, v = self.att_proj(self.attn_norm(x)).view(B, S, 3, self.h, C // self.h).permute(2, 0, 3, 1, 4)
        q, k = apply_rope(q.float(), cos, sin).to(v.dtype), apply_rope(k.float(), cos, sin).to(v.dtype)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.attn_out(a.transpose(1, 2).reshape(B, S, C)).to(x.dtype)
        val, gate = self.ff_proj(self.ff_norm(x)).chunk(2, dim=-1)
        return x + self.ff_out(F.silu(gate) * val).to(x.dtype)


class OLMo(Module):
    """OLMo-150M shape (olmo.rs): d 768, 12 layers, 12 heads, RMSNorm eps 1e-6,
    SwiGLU with mlp_ratio 8 (effective 4 d), RoPE, no biases, no weight tying,
    vocab 50,280 padded to 50,304."""

    NAME = "olmo"

    def __init__(self, vocab=50304, d=768, layers=12, heads=12, mlp_ratio=8, max_seq=256,
                 device=None):
        super().__init__()
        self.emb = Embedding(vocab, d, device=device)
        self.blocks = torch.nn.ModuleList(
            [OLMoBlock(d, heads, mlp_ratio * d // 2, device) for _ in range(layers)])
        self.norm = RMSNorm(d, eps=1e-6, device=device)
        self.head = Linear(d, vocab, bias=False, device=device)
        self.heads, self.max_seq = heads, max_seq

    def forward(self, ids):
        x = self.emb(ids).float()
        cos, sin = rope_cache(ids.shape[1], x.shape[-1] // self.heads, device=x.device)
        for b in self.blocks:
            x = b(x, cos, sin)
        return self.head(self.norm(x))


def _olmo_small(device):
    return OLMo(vocab=512, d=128, layers=2, heads=2, max_seq=64, device=device)


# ------------------------------------------------------------------ registry
ZOO: Dict[str, ModelDef] = {
    "logistic": ModelDef("logistic", "Logistic regression on MNIST (~92% acc)", _logistic,
                         lambda n=1024: _images(n, (1, 28, 28), 10), _ce,
                         lambda p, lr: Adam(p, lr)),
    "mlp": ModelDef("mlp", "2-layer MLP on MNIST (~97% acc)", _mlp,
                    lambda n=1024: _images(n, (1, 28, 28), 10), _ce, lambda p, lr: Adam(p, lr)),
    "lenet": ModelDef("lenet", "LeNet-5 on MNIST (~99% acc, LeCun 1998)", _lenet,
                      lambda n=1024: _images(n, (1, 28, 28), 10), _ce, lambda p, lr: Adam(p, lr)),
    "conv_ae": ModelDef("conv_ae", "Conv autoencoder on MNIST", _conv_ae,
                        lambda n=1024: _images(n, (1, 28, 28), 10), _recon,
                        lambda p, lr: Adam(p, lr)),
    "char_rnn": ModelDef("char_rnn", "Char-RNN (2-layer LSTM) on Shakespeare", lambda d: CharRNN(device=d),
                         lambda n=256: _chars(n, 128, 65), _seq_ce, lambda p, lr: RMSprop(p, lr),
                         lr=2e-3),
    "gpt_nano": ModelDef("gpt_nano", "GPT-nano on Shakespeare (4 layers, 4 heads, d 128)", _gpt_nano,
                         lambda n=256: _chars(n, 128, 65), _lm_loss, lambda p, lr: Adam(p, lr),
                         lr=3e-4),
    "resnet": ModelDef("resnet", "ResNet-20 on CIFAR-10 (He et al. 2015)",
                       lambda d: __import__("flodl_b200.models.resnet", fromlist=["ResNet20"]).ResNet20(device=d),
                       lambda n=512: _images(n, (3, 32, 32), 10),
                       lambda m, b: m.loss(b[0], b[1]),
                       lambda p, lr: SGD(p, lr, momentum=0.9, weight_decay=1e-4), lr=0.1),
    "olmo": ModelDef("olmo", "OLMo-150M-style decoder (RMSNorm, RoPE, SwiGLU)", lambda d: OLMo(device=d),
                     lambda n=64: _chars(n, 256, 50280), _seq_ce,
                     lambda p, lr: AdamW(p, lr, weight_decay=0.1), batch_size=4, lr=6e-4),
    "olmo_small": ModelDef("olmo_small", "OLMo-style decoder, test size", _olmo_small,
                           lambda n=64: _chars(n, 64, 512), _seq_ce,
                           lambda p, lr: AdamW(p, lr, weight_decay=0.1), batch_size=8, lr=1e-3),
}
