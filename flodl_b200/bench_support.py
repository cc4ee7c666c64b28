"""Step builders for bench.py: the framework arm and a stock-PyTorch proxy arm.

Each benchmark model is described by a :class:`BenchModel`
with its per-GPU batch, sequence length, description and two builders:

* ``flodl(dev, world, engine)`` - this framework: fused whole-model training
  op, flat parameter arenas, fused peer-memory all-reduce + optimizer (or NCCL
  buckets with ``engine="nccl"``).
* ``torch(dev, world)`` - the same model in stock PyTorch (cuBLAS / cuDNN /
  SDPA kernels under bf16 autocast, fused AdamW, NCCL DDP).

A builder returns ``(step, state)``: ``step()`` runs one full training step on
the static device inputs ``state["inputs"]`` and returns the loss tensor;
``state["host_inputs"]()`` makes pinned host tensors of the same shapes (the
end-to-end run copies them in every step).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict

import torch
import torch.nn.functional as F


@dataclass
class BenchModel:
    name: str
    desc: str
    batch: int       # per GPU
    seq: int         # tokens per sample (1 for image models)
    optimizer: str
    flodl: Callable
    torch: Callable


def _pinned_like(ts, gen_fn):
    def make():
        return [gen_fn(i, t).pin_memory() for i, t in enumerate(ts)]
    return make


# --------------------------------------------------------------------------- LM (config 3)
LM_B, LM_S, LM_V = 64, 256, 256


def _lm_flodl(dev, world, engine):
    from .models import TransformerLM
    from .optim import AdamW
    from .parallel.ddp import Ddp

    model = TransformerLM(vocab_size=LM_V, d_model=512, n_layers=6, n_heads=8, d_ff=2048,
                          max_seq=LM_S, device=dev)
    ddp = None
    if engine == "peer":
        from .parallel.fused import FusedDdp
        opt = AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
        ddp = FusedDdp(model, opt)
    elif world > 1:
        ddp = Ddp(model, engine="nccl")
        opt = AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
    else:
        opt = AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    ids = torch.randint(0, LM_V, (LM_B, LM_S), device=dev, generator=g)
    tgt = torch.randint(0, LM_V, (LM_B, LM_S), device=dev, generator=g)
    step = _make_step(lambda: model.loss(ids, tgt), ddp, opt)
    host = _pinned_like([ids, tgt], lambda i, t: torch.randint(0, LM_V, tuple(t.shape)))
    return step, {"inputs": [ids, tgt], "host_inputs": host, "model": model, "opt": opt,
                  "ddp": ddp}


class _TorchBlock(torch.nn.Module):
    def __init__(self, d, h, f):
        super().__init__()
        self.h = h
        self.ln1 = torch.nn.LayerNorm(d)
        self.qkv = torch.nn.Linear(d, 3 * d)
        self.proj = torch.nn.Linear(d, d)
        self.ln2 = torch.nn.LayerNorm(d)
        self.fc1 = torch.nn.Linear(d, f)
        self.fc2 = torch.nn.Linear(f, d)

    def forward(self, x):
        B, S, C = x.shape
        q, k, v = self.qkv(self.ln1(x)).view(B, S, 3, self.h, C // self.h).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.proj(a.transpose(1, 2).reshape(B, S, C))
        return x + self.fc2(F.gelu(self.fc1(self.ln2(x))))


class _TorchLM(torch.nn.Module):
    def __init__(self, V, d, L, h, f, S):
        super().__init__()
        self.tok = torch.nn.Embedding(V, d)
        self.pos = torch.nn.Parameter(torch.randn(S, d) * 0.02)
        self.blocks = torch.nn.ModuleList([_TorchBlock(d, h, f) for _ in range(L)])
        self.ln = torch.nn.LayerNorm(d)
        self.head = torch.nn.Linear(d, V)

    def forward(self, ids, tgt):
        x = self.tok(ids) + self.pos[: ids.shape[1]]
        for b in self.blocks:
            x = b(x)
        logits = self.head(self.ln(x))
        return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), tgt.reshape(-1))


def _lm_torch(dev, world):
    model = _TorchLM(LM_V, 512, 6, 8, 2048, LM_S).to(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    ids = torch.randint(0, LM_V, (LM_B, LM_S), device=dev, generator=g)
    tgt = torch.randint(0, LM_V, (LM_B, LM_S), device=dev, generator=g)
    step, model, opt = _torch_step(model, dev, world, lambda m: m(ids, tgt), "adamw")
    host = _pinned_like([ids, tgt], lambda i, t: torch.randint(0, LM_V, tuple(t.shape)))
    return step, {"inputs": [ids, tgt], "host_inputs": host, "model": model, "opt": opt}


# --------------------------------------------------------------------------- BERT (config 4)
BERT_B, BERT_S, BERT_V = 32, 512, 30522
BERT_MASKED = int(0.15 * BERT_S + 0.5)  # masked positions per sequence


def _bert_batch(dev, gen=None):
    kw = {"generator": gen} if gen is not None else {}
    d = dev if gen is not None else "cpu"
    ids = torch.randint(0, BERT_V, (BERT_B, BERT_S), device=d, **kw)
    scores = torch.rand(BERT_B, BERT_S, device=d, **kw)
    pos = scores.topk(BERT_MASKED, dim=1).indices
    labels = torch.full((BERT_B, BERT_S), -100, dtype=torch.int64, device=d)
    labels.scatter_(1, pos, ids.gather(1, pos))
    return ids, labels


def _bert_flodl(dev, world, engine):
    from .models.bert import BertConfig, BertForMaskedLM
    from .optim import AdamW
    from .parallel.ddp import Ddp

    model = BertForMaskedLM(BertConfig.bert_base_uncased(), device=dev)
    ddp = None
    if engine == "peer":
        from .parallel.fused import FusedDdp
        opt = AdamW(model.parameters(), lr=1e-4, weight_decay=0.01)
        ddp = FusedDdp(model, opt)
    elif world > 1:
        ddp = Ddp(model, engine="nccl")
        opt = AdamW(model.parameters(), lr=1e-4, weight_decay=0.01)
    else:
        opt = AdamW(model.parameters(), lr=1e-4, weight_decay=0.01)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    ids, labels = _bert_batch(dev, g)
    rows = BERT_B * BERT_MASKED
    step = _make_step(lambda: model.loss(ids, labels, masked_rows=rows), ddp, opt)

    def host():
        a, b = _bert_batch("cpu")
        return [a.pin_memory(), b.pin_memory()]

    return step, {"inputs": [ids, labels], "host_inputs": host, "model": model, "opt": opt,
                  "ddp": ddp}


def _bert_torch(dev, world):
    from transformers import BertConfig as HFConfig
    from transformers import BertForMaskedLM as HFBert

    cfg = HFConfig(attn_implementation="sdpa")
    model = HFBert(cfg).to(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    ids, labels = _bert_batch(dev, g)
    step, model, opt = _torch_step(model, dev, world,
                                   lambda m: m(input_ids=ids, labels=labels).loss, "adamw",
                                   lr=1e-4, wd=0.01)

    def host():
        a, b = _bert_batch("cpu")
        return [a.pin_memory(), b.pin_memory()]

    return step, {"inputs": [ids, labels], "host_inputs": host, "model": model, "opt": opt}


# --------------------------------------------------------------------------- ResNet-20 (config 2)
RN_B = 128


def _rn_batch(dev, gen=None):
    kw = {"generator": gen} if gen is not None else {}
    d = dev if gen is not None else "cpu"
    x = torch.randn(RN_B, 3, 32, 32, device=d, **kw)
    y = torch.randint(0, 10, (RN_B,), device=d, **kw)
    return x, y


def _rn_flodl(dev, world, engine):
    from .models import ResNet20
    from .optim import SGD
    from .parallel.ddp import Ddp

    model = ResNet20(device=dev)
    ddp = None
    mk = lambda: SGD(model.parameters(), lr=0.1, momentum=0.9, weight_decay=1e-4)
    if engine == "peer":
        from .parallel.fused import FusedDdp
        opt = mk()
        ddp = FusedDdp(model, opt)
    elif world > 1:
        ddp = Ddp(model, engine="nccl")
        opt = mk()
    else:
        opt = mk()
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    x, y = _rn_batch(dev, g)
    step = _make_step(lambda: model.loss(x, y), ddp, opt)

    def host():
        a, b = _rn_batch("cpu")
        return [a.pin_memory(), b.pin_memory()]

    return step, {"inputs": [x, y], "host_inputs": host, "model": model, "opt": opt, "ddp": ddp}


class _TorchBlock2(torch.nn.Module):
    def __init__(self, cin, cout, stride):
        super().__init__()
        nn = torch.nn
        self.c1 = nn.Conv2d(cin, cout, 3, stride, 1, bias=False)
        self.b1 = nn.BatchNorm2d(cout)
        self.c2 = nn.Conv2d(cout, cout, 3, 1, 1, bias=False)
        self.b2 = nn.BatchNorm2d(cout)
        self.ds = (nn.Sequential(nn.Conv2d(cin, cout, 1, stride, bias=False), nn.BatchNorm2d(cout))
                   if stride != 1 or cin != cout else None)

    def forward(self, x):
        idn = self.ds(x) if self.ds is not None else x
        return F.relu(self.b2(self.c2(F.relu(self.b1(self.c1(x))))) + idn)


class _TorchResNet20(torch.nn.Module):
    def __init__(self):
        super().__init__()
        nn = torch.nn
        self.c = nn.Conv2d(3, 16, 3, 1, 1, bias=False)
        self.b = nn.BatchNorm2d(16)
        blocks = []
        for cin, cout, s in ((16, 16, 1), (16, 32, 2), (32, 64, 2)):
            blocks += [_TorchBlock2(cin, cout, s), _TorchBlock2(cout, cout, 1),
                       _TorchBlock2(cout, cout, 1)]
        self.blocks = nn.Sequential(*blocks)
        self.fc = nn.Linear(64, 10)

    def forward(self, x, y):
        h = self.blocks(F.relu(self.b(self.c(x))))
        return F.cross_entropy(self.fc(F.adaptive_avg_pool2d(h, 1).flatten(1)).float(), y)


def _rn_torch(dev, world):
    model = _TorchResNet20().to(dev).to(memory_format=torch.channels_last)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    x, y = _rn_batch(dev, g)
    step, model, opt = _torch_step(model, dev, world, lambda m: m(x, y), "sgd", lr=0.1, wd=1e-4)

    def host():
        a, b = _rn_batch("cpu")
        return [a.pin_memory(), b.pin_memory()]

    return step, {"inputs": [x, y], "host_inputs": host, "model": model, "opt": opt}


# --------------------------------------------------------------------------- shared
def _make_step(loss_fn, ddp, opt):
    if ddp is not None and getattr(ddp, "fuses_optimizer", False):
        def step():
            loss = loss_fn()
            loss.backward()
            ddp.finish()
            return loss
    else:
        def step():
            loss = loss_fn()
            loss.backward()
            if ddp is not None:
                ddp.finish()
            opt.step()
            opt.zero_grad()
            return loss
    return step


def _torch_step(model, dev, world, loss_of, opt_kind, lr=3e-4, wd=0.1, momentum=0.9):
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[dev.index],
                                                          gradient_as_bucket_view=True)
    if opt_kind == "adamw":
        opt = torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=wd, fused=True,
                                capturable=True)
    else:
        opt = torch.optim.SGD(model.parameters(), lr=lr, momentum=momentum, weight_decay=wd)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = loss_of(model)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=False)
        return loss

    return step, model, opt


MODELS: Dict[str, BenchModel] = {
    "lm": BenchModel("lm", "transformer-lm 6L d512 h8 ff2048 vocab256 pre-LN GELU", LM_B, LM_S,
                     "AdamW lr3e-4 wd0.1", _lm_flodl, _lm_torch),
    "bert": BenchModel("bert", "bert-base MLM 12L d768 h12 ff3072 vocab30522 (15% masked)",
                       BERT_B, BERT_S, "AdamW lr1e-4 wd0.01", _bert_flodl, _bert_torch),
    "resnet20": BenchModel("resnet20", "resnet-20 CIFAR (3x3 basic blocks 16/32/64, BN, ReLU), 3x32x32",
                           RN_B, 1, "SGD lr0.1 momentum0.9 wd1e-4", _rn_flodl, _rn_torch),
}
