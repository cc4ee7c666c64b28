"""Step builders for bench.py: the framework arm and a stock-PyTorch proxy arm."""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def flodl_arm_step(dev, world, B, S, V, engine):
    from .models import TransformerLM
    from .optim import AdamW
    from .parallel.ddp import Ddp

    model = TransformerLM(vocab_size=V, d_model=512, n_layers=6, n_heads=8, d_ff=2048, max_seq=S,
                          device=dev)
    ddp = None
    if world > 1:
        if engine == "peer":
            from .parallel.fused import FusedDdp
            opt = AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
            ddp = FusedDdp(model, opt)
        else:
            ddp = Ddp(model, engine="nccl")
            opt = AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
    else:
        opt = AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    ids = torch.randint(0, V, (B, S), device=dev, generator=g)
    tgt = torch.randint(0, V, (B, S), device=dev, generator=g)

    if ddp is not None and getattr(ddp, "fuses_optimizer", False):
        def step():
            loss = model.loss(ids, tgt)
            loss.backward()
            ddp.finish()
            return loss
    else:
        def step():
            loss = model.loss(ids, tgt)
            loss.backward()
            if ddp is not None:
                ddp.finish()
            opt.step()
            opt.zero_grad()
            return loss

    return step, {"ids": ids, "tgt": tgt, "model": model, "opt": opt, "ddp": ddp}


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


def torch_arm_step(dev, world, B, S, V):
    """Stock PyTorch: autocast bf16, cuBLAS/SDPA kernels, fused AdamW, NCCL DDP."""
    model = _TorchLM(V, 512, 6, 8, 2048, S).to(dev)
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[dev.index],
                                                          gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.1, fused=True,
                            capturable=True)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    ids = torch.randint(0, V, (B, S), device=dev, generator=g)
    tgt = torch.randint(0, V, (B, S), device=dev, generator=g)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(ids, tgt)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=False)
        return loss

    return step, {"ids": ids, "tgt": tgt, "model": model, "opt": opt}
