"""Model benchmark suite: this framework vs plain PyTorch on the same models.

Reference: benchmarks/src/{harness.rs, tier1/*, tier2/*} and
benchmarks/python/*. Eleven models with the reference's shapes, optimiser
(Adam 1e-3), synthetic data and harness:

* tier 1 - mlp (1024-2048x4-1024, B 256), convnet (5 conv/BN/ReLU/maxpool
  blocks on 3x64x64, B 128), conv_autoencoder (4 strided convs + 4 transposed
  convs, B 64), gru_seq (GRUCell unrolled over 50 steps, 256->512, B 128),
  lstm_seq (2-layer LSTM over 50 steps, B 128), transformer (4 post-LN encoder
  layers, d 512, 8 heads, FFN 2048, vocab 8192, seq 128, B 32);
* tier 2 (graph control flow) - feedback_loop (residual body until a learned
  halt, <= 10 iterations), feedback_loop_fixed (10 iterations),
  gated_routing (soft gate over 8 experts, B 256), iterative_refine (8
  refinement passes, d 1024), residual_tower (12 residual blocks, d 1024).

Harness: ``runs`` passes (the first one discarded as warm-up), each with
``warmup_epochs`` untimed and ``measured_epochs`` timed epochs of
``batches_per_epoch`` steps (forward, loss, backward, Adam step); the
reported epoch times are those of the pass with the lowest median, and the
per-pass medians are kept for spread. Epochs are timed with CUDA events on
the device (host clock on CPU).

Arms: ``flodl`` builds the model from this package (FlowBuilder graphs, its
layers, its sm_100a kernels on CUDA - bf16 tensor-core GEMMs with f32
accumulation and f32 master weights); ``flodl-graph`` is the same model with
the whole training step (forward, loss, backward, optimizer) captured once as
a CUDA graph and replayed (``StepRunner.capture_training``; models with
host-side control flow cannot be captured and report so); ``torch`` builds the
same model from ``torch.nn`` in f32; ``torch-bf16`` runs that under bf16
autocast, the precision-matched baseline.

    python -m flodl_b200.benchmarks [--models mlp,transformer] [--arms flodl,torch]
                                    [--runs 4] [--warmup 3] [--epochs 20] [--scale 1.0]
"""
from __future__ import annotations

import argparse
import contextlib
import json
import statistics
import time
from dataclasses import asdict, dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.nn as tnn
import torch.nn.functional as F


@dataclass
class BenchConfig:
    name: str
    batch_size: int = 128
    batches_per_epoch: int = 50
    runs: int = 4
    warmup_epochs: int = 3
    measured_epochs: int = 20


@dataclass
class BenchResult:
    name: str
    arm: str
    device: str
    runs: int
    warmup_epochs: int
    measured_epochs: int
    batches_per_epoch: int
    batch_size: int
    param_count: int
    epoch_times_ms: List[float] = field(default_factory=list)
    median_epoch_ms: float = 0.0
    mean_epoch_ms: float = 0.0
    min_epoch_ms: float = 0.0
    max_epoch_ms: float = 0.0
    run_medians_ms: List[float] = field(default_factory=list)
    final_loss: float = 0.0
    vram_mb: Optional[float] = None


# ----------------------------------------------------------------- model builders
def _S(n, scale):
    return max(1, int(round(n * scale)))


def _mlp(arm, dev, s):
    D, Hd = _S(1024, s), _S(2048, s)
    dims = [D, Hd, Hd, Hd, Hd, D]
    if arm == "flodl":
        from .graph import FlowBuilder
        from .nn import GELU, LayerNorm, Linear
        b = FlowBuilder.from_(Linear(dims[0], dims[1], device=dev))
        for i in range(1, 5):
            b = b.through(GELU()).through(LayerNorm(dims[i], device=dev)).through(
                Linear(dims[i], dims[i + 1], device=dev))
        m = b.build()
    else:
        layers = [tnn.Linear(dims[0], dims[1])]
        for i in range(1, 5):
            layers += [tnn.GELU(), tnn.LayerNorm(dims[i]), tnn.Linear(dims[i], dims[i + 1])]
        m = tnn.Sequential(*layers).to(dev)
    data = lambda B: (torch.randn(B, D, device=dev), torch.randn(B, D, device=dev))
    return m, data, F.mse_loss


def _convnet(arm, dev, s):
    ch = [3, _S(64, s), _S(128, s), _S(256, s), _S(512, s), _S(512, s)]
    if arm == "flodl":
        from .graph import FlowBuilder
        from .nn import AdaptiveAvgPool2d, BatchNorm2d, Conv2d, Flatten, Linear, MaxPool2d, ReLU
        b = FlowBuilder.from_(Conv2d(3, ch[1], 3, padding=1, device=dev))
        for i in range(1, 6):
            if i > 1:
                b = b.through(Conv2d(ch[i - 1], ch[i], 3, padding=1, device=dev))
            b = b.through(BatchNorm2d(ch[i], device=dev)).through(ReLU())
            if i < 5:
                b = b.through(MaxPool2d(2))
        m = b.through(AdaptiveAvgPool2d(1)).through(Flatten()).through(Linear(ch[5], 100, device=dev)).build()
    else:
        layers = []
        for i in range(1, 6):
            layers += [tnn.Conv2d(ch[i - 1], ch[i], 3, padding=1), tnn.BatchNorm2d(ch[i]), tnn.ReLU()]
            if i < 5:
                layers.append(tnn.MaxPool2d(2))
        layers += [tnn.AdaptiveAvgPool2d(1), tnn.Flatten(), tnn.Linear(ch[5], 100)]
        m = tnn.Sequential(*layers).to(dev)
    data = lambda B: (torch.randn(B, 3, 64, 64, device=dev), torch.randn(B, 100, device=dev))
    return m, data, F.mse_loss


def _conv_ae(arm, dev, s):
    ch = [3, _S(64, s), _S(128, s), _S(256, s), _S(512, s)]
    if arm == "flodl":
        from .graph import FlowBuilder
        from .nn import BatchNorm2d, Conv2d, ConvTranspose2d, ReLU, Tanh
        b = FlowBuilder.from_(Conv2d(3, ch[1], 4, stride=2, padding=1, device=dev))
        for i in range(1, 5):
            if i > 1:
                b = b.through(Conv2d(ch[i - 1], ch[i], 4, stride=2, padding=1, device=dev))
            b = b.through(BatchNorm2d(ch[i], device=dev)).through(ReLU())
        for i in range(4, 1, -1):
            b = (b.through(ConvTranspose2d(ch[i], ch[i - 1], 4, stride=2, padding=1, device=dev))
                 .through(BatchNorm2d(ch[i - 1], device=dev)).through(ReLU()))
        m = b.through(ConvTranspose2d(ch[1], 3, 4, stride=2, padding=1, device=dev)).through(Tanh()).build()
    else:
        layers = []
        for i in range(1, 5):
            layers += [tnn.Conv2d(ch[i - 1], ch[i], 4, 2, 1), tnn.BatchNorm2d(ch[i]), tnn.ReLU()]
        for i in range(4, 1, -1):
            layers += [tnn.ConvTranspose2d(ch[i], ch[i - 1], 4, 2, 1), tnn.BatchNorm2d(ch[i - 1]), tnn.ReLU()]
        layers += [tnn.ConvTranspose2d(ch[1], 3, 4, 2, 1), tnn.Tanh()]
        m = tnn.Sequential(*layers).to(dev)

    def data(B):
        x = torch.randn(B, 3, 64, 64, device=dev)
        return x, x
    return m, data, F.mse_loss


class _TorchGruSeq(tnn.Module):
    def __init__(self, i, h):
        super().__init__()
        self.cell, self.out = tnn.GRUCell(i, h), tnn.Linear(h, i)

    def forward(self, x):
        h = None
        for t in range(x.shape[1]):
            h = self.cell(x[:, t], h)
        return self.out(h)


def _gru_seq(arm, dev, s):
    I, Hd, T = _S(256, s), _S(512, s), max(2, _S(50, s))
    if arm == "flodl":
        from .nn import GRUCell, Linear
        from .nn.module import Module

        class GruSeq(Module):
            NAME = "gru_seq"

            def __init__(self):
                super().__init__()
                self.cell, self.out = GRUCell(I, Hd, device=dev), Linear(Hd, I, device=dev)

            def forward(self, x):
                self.cell.reset()  # the cell keeps state across calls; each batch starts fresh
                h = None
                for t in range(x.shape[1]):
                    h = self.cell(x[:, t], h)
                return self.out(h)
        m = GruSeq()
    else:
        m = _TorchGruSeq(I, Hd).to(dev)
    data = lambda B: (torch.randn(B, T, I, device=dev), torch.randn(B, I, device=dev))
    return m, data, F.mse_loss


class _TorchLstmSeq(tnn.Module):
    def __init__(self, i, h):
        super().__init__()
        self.lstm, self.out = tnn.LSTM(i, h, 2, batch_first=True), tnn.Linear(h, i)

    def forward(self, x):
        return self.out(self.lstm(x)[0][:, -1])


def _lstm_seq(arm, dev, s):
    I, Hd, T = _S(256, s), _S(512, s), max(2, _S(50, s))
    if arm == "flodl":
        from .nn import LSTM, Linear
        from .nn.module import Module

        class LstmSeq(Module):
            NAME = "lstm_seq"

            def __init__(self):
                super().__init__()
                self.lstm = LSTM(I, Hd, 2, batch_first=True, device=dev)
                self.out = Linear(Hd, I, device=dev)

            def forward(self, x):
                self.lstm.reset()
                return self.out(self.lstm(x)[:, -1])
        m = LstmSeq()
    else:
        m = _TorchLstmSeq(I, Hd).to(dev)
    data = lambda B: (torch.randn(B, T, I, device=dev), torch.randn(B, I, device=dev))
    return m, data, F.mse_loss


class _TorchEncoder(tnn.Module):
    def __init__(self, V, d, h, ff, L, S):
        super().__init__()
        self.emb = tnn.Embedding(V, d)
        self.pos = tnn.Parameter(torch.randn(1, S, d))
        self.layers = tnn.ModuleList([tnn.TransformerEncoderLayer(d, h, ff, 0.0, "gelu", batch_first=True)
                                      for _ in range(L)])
        self.out = tnn.Linear(d, V)

    def forward(self, ids):
        x = self.emb(ids) + self.pos
        for l in self.layers:
            x = l(x)
        return self.out(x)


def _transformer(arm, dev, s):
    V, d, ff, H, L, S = _S(8192, s), _S(512, s), _S(2048, s), 8, 4, max(8, _S(128, s))
    d = max(H * 8, d // H * H)
    if arm == "flodl":
        from .nn import GELU, Embedding, LayerNorm, Linear, MultiheadAttention
        from .nn.module import Module

        class Layer(Module):
            NAME = "encoder_layer"

            def __init__(self):
                super().__init__()
                self.mha = MultiheadAttention(d, H, device=dev)
                self.norm1, self.norm2 = LayerNorm(d, device=dev), LayerNorm(d, device=dev)
                self.ff1, self.ff2 = Linear(d, ff, device=dev), Linear(ff, d, device=dev)
                self.act = GELU()

            def forward(self, x):
                x = self.norm1(x + self.mha(x).to(x.dtype))
                return self.norm2(x + self.ff2(self.act(self.ff1(x))).to(x.dtype))

        class Encoder(Module):
            NAME = "transformer"

            def __init__(self):
                super().__init__()
                self.emb = Embedding(V, d, device=dev)
                self.pos = torch.nn.Parameter(torch.randn(1, S, d, device=dev))
                self.layers = torch.nn.ModuleList([Layer() for _ in range(L)])
                self.out = Linear(d, V, device=dev)

            def forward(self, ids):
                x = self.emb(ids).float() + self.pos
                for l in self.layers:
                    x = l(x)
                return self.out(x)
        m = Encoder()
    else:
        m = _TorchEncoder(V, d, H, ff, L, S).to(dev)

    def data(B):
        return (torch.randint(0, V, (B, S), device=dev), torch.randint(0, V, (B, S), device=dev))

    def loss(logits, y):
        return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), y.reshape(-1))
    return m, data, loss


def _residual_block_flodl(D, dev):
    from .graph import FlowBuilder
    from .nn import GELU, LayerNorm, Linear
    return FlowBuilder.from_(Linear(D, D, device=dev)).through(GELU()).through(LayerNorm(D, device=dev)).build()


class _TorchResBody(tnn.Module):
    def __init__(self, D):
        super().__init__()
        self.f = tnn.Sequential(tnn.Linear(D, D), tnn.GELU(), tnn.LayerNorm(D))

    def forward(self, x):
        return x + self.f(x)


def _halt_init(lin) -> None:
    """Both arms start from the same halting head (zero weights, bias -2:
    sigmoid < 0.5, so every forward runs all iterations; the halting decision
    is not differentiable, so it stays that way). Random heads would make the
    two arms run different iteration counts and time different work."""
    with torch.no_grad():
        lin.weight.zero_()
        lin.bias.fill_(-2.0)


class _TorchLoopModel(tnn.Module):
    def __init__(self, D, iters, halt):
        super().__init__()
        self.enc = tnn.Sequential(tnn.Linear(D, D), tnn.GELU(), tnn.LayerNorm(D))
        self.body, self.iters = _TorchResBody(D), iters
        self.halt = tnn.Linear(D, 1) if halt else None
        if self.halt is not None:
            _halt_init(self.halt)
        self.dec = tnn.Linear(D, D)

    def forward(self, x):
        x = self.enc(x)
        for _ in range(self.iters):
            x = self.body(x)
            # the same learned halting rule as the graph arm: mean sigmoid(Wx) - 0.5 > 0
            if self.halt is not None and float(torch.sigmoid(self.halt(x)).mean()) - 0.5 > 0:
                break
        return self.dec(x)


def _loop_model(arm, dev, s, D0, iters, halt):
    D = _S(D0, s)
    if arm == "flodl":
        from .graph import FlowBuilder, LearnedHalt
        from .nn import GELU, LayerNorm, Linear
        body = FlowBuilder.new().also(_residual_block_flodl(D, dev)).build()
        b = (FlowBuilder.from_(Linear(D, D, device=dev)).through(GELU()).through(LayerNorm(D, device=dev))
             .loop_body(body))
        if halt:
            lh = LearnedHalt(D, device=dev)
            _halt_init(lh.proj)
            b = b.until_cond(lh, iters)
        else:
            b = b.for_n(iters)
        m = b.through(Linear(D, D, device=dev)).build()
    else:
        m = _TorchLoopModel(D, iters, halt).to(dev)
    data = lambda B: (torch.randn(B, D, device=dev), torch.randn(B, D, device=dev))
    return m, data, F.mse_loss


class _TorchGate(tnn.Module):
    def __init__(self, D, E):
        super().__init__()
        self.inp = tnn.Sequential(tnn.Linear(D, D), tnn.GELU())
        self.router = tnn.Linear(D, E)
        self.experts = tnn.ModuleList([tnn.Sequential(tnn.Linear(D, D), tnn.GELU(), tnn.LayerNorm(D))
                                       for _ in range(E)])
        self.out = tnn.Linear(D, D)

    def forward(self, x):
        x = self.inp(x)
        w = torch.softmax(self.router(x), -1)
        y = sum(e(x) * w[:, i:i + 1] for i, e in enumerate(self.experts))
        return self.out(y)


def _gated(arm, dev, s):
    D, E = _S(512, s), 8
    if arm == "flodl":
        from .graph import FlowBuilder, SoftmaxRouter
        from .nn import GELU, Linear
        m = (FlowBuilder.from_(Linear(D, D, device=dev)).through(GELU())
             .gate(SoftmaxRouter(D, E, device=dev), [_residual_block_flodl(D, dev) for _ in range(E)])
             .through(Linear(D, D, device=dev)).build())
    else:
        m = _TorchGate(D, E).to(dev)
    data = lambda B: (torch.randn(B, D, device=dev), torch.randn(B, D, device=dev))
    return m, data, F.mse_loss


class _TorchTower(tnn.Module):
    def __init__(self, D, n):
        super().__init__()
        self.inp = tnn.Linear(D, D)
        self.blocks = tnn.ModuleList([_TorchResBody(D) for _ in range(n)])
        self.out = tnn.Linear(D, D)

    def forward(self, x):
        x = self.inp(x)
        for b in self.blocks:
            x = b(x)
        return self.out(x)


def _tower(arm, dev, s):
    D, n = _S(1024, s), 12
    if arm == "flodl":
        from .graph import FlowBuilder
        from .nn import Linear
        b = FlowBuilder.from_(Linear(D, D, device=dev))
        for _ in range(n):
            b = b.also(_residual_block_flodl(D, dev))
        m = b.through(Linear(D, D, device=dev)).build()
    else:
        m = _TorchTower(D, n).to(dev)
    data = lambda B: (torch.randn(B, D, device=dev), torch.randn(B, D, device=dev))
    return m, data, F.mse_loss


SUITE: Dict[str, Tuple[BenchConfig, Callable]] = {
    "mlp": (BenchConfig("mlp", 256), _mlp),
    "convnet": (BenchConfig("convnet", 128), _convnet),
    "conv_autoencoder": (BenchConfig("conv_autoencoder", 64), _conv_ae),
    "gru_seq": (BenchConfig("gru_seq", 128), _gru_seq),
    "lstm_seq": (BenchConfig("lstm_seq", 128), _lstm_seq),
    "transformer": (BenchConfig("transformer", 32), _transformer),
    "feedback_loop": (BenchConfig("feedback_loop", 128),
                      lambda a, d, s: _loop_model(a, d, s, 512, 10, True)),
    "feedback_loop_fixed": (BenchConfig("feedback_loop_fixed", 128),
                            lambda a, d, s: _loop_model(a, d, s, 512, 10, False)),
    "gated_routing": (BenchConfig("gated_routing", 256), _gated),
    "iterative_refine": (BenchConfig("iterative_refine", 256),
                         lambda a, d, s: _loop_model(a, d, s, 1024, 8, False)),
    "residual_tower": (BenchConfig("residual_tower", 256), _tower),
}


# ----------------------------------------------------------------- harness
def _optimizer(arm, params):
    params = list(params)
    if arm.startswith("flodl"):
        from .optim import Adam
        return Adam(params, lr=1e-3)
    return torch.optim.Adam(params, lr=1e-3)


def run_benchmark(name: str, arm: str = "flodl", device: Optional[str] = None, runs: int = 4,
                  warmup_epochs: int = 3, measured_epochs: int = 20,
                  batches_per_epoch: Optional[int] = None, scale: float = 1.0,
                  batch_scale: float = 1.0, seed: int = 0) -> BenchResult:
    cfg, build = SUITE[name]
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    torch.manual_seed(seed)
    model, data, loss_fn = build("flodl" if arm.startswith("flodl") else "torch", dev, scale)
    model.train()
    opt = _optimizer(arm, model.parameters())
    B = max(1, int(cfg.batch_size * batch_scale))
    nb = batches_per_epoch or cfg.batches_per_epoch
    batches = [data(B) for _ in range(nb)]
    amp = (torch.autocast(dev.type, dtype=torch.bfloat16) if arm == "torch-bf16"
           else contextlib.nullcontext())
    cuda = dev.type == "cuda"

    runner = None
    if arm == "flodl-graph":
        if not cuda:
            raise RuntimeError("flodl-graph needs CUDA")
        from .train import StepRunner

        def lf(out, y):
            return loss_fn(out.float(), y) if y.is_floating_point() else loss_fn(out, y)
        runner = StepRunner.capture_training(model, opt, lf, list(batches[0]))

    def epoch() -> Tuple[float, float]:
        total = torch.zeros((), device=dev)
        if runner is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for x, y in batches:
                total += runner.replay(x, y)
            e1.record()
            e1.synchronize()
            return e0.elapsed_time(e1), float(total) / nb
        if cuda:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        t0 = time.perf_counter()
        for x, y in batches:
            with amp:
                out = model(x)
            loss = loss_fn(out.float(), y) if y.is_floating_point() else loss_fn(out, y)
            loss.backward()
            opt.step()
            opt.zero_grad()
            total += loss.detach()
        if cuda:
            e1.record()
            e1.synchronize()
            ms = e0.elapsed_time(e1)
        else:
            ms = (time.perf_counter() - t0) * 1e3
        return ms, float(total) / nb

    def one_pass():
        for _ in range(warmup_epochs):
            epoch()
        times, loss = [], 0.0
        for _ in range(measured_epochs):
            ms, loss = epoch()
            times.append(ms)
        return times, loss

    one_pass()  # warm-up pass, discarded
    if cuda:
        torch.cuda.reset_peak_memory_stats(dev)
    best, medians, final = None, [], 0.0
    for _ in range(max(2, runs) - 1):
        times, final = one_pass()
        med = statistics.median(times)
        medians.append(med)
        if best is None or med < statistics.median(best):
            best = times
    r = BenchResult(name, arm, f"CUDA ({torch.cuda.get_device_name(dev)})" if cuda else "CPU",
                    runs, warmup_epochs, measured_epochs, nb, B,
                    sum(p.numel() for p in model.parameters()), best, statistics.median(best),
                    statistics.mean(best), min(best), max(best), medians, final,
                    torch.cuda.max_memory_allocated(dev) / 2 ** 20 if cuda else None)
    return r


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--models", default=",".join(SUITE))
    ap.add_argument("--arms", default="flodl,torch,torch-bf16,flodl-graph")
    ap.add_argument("--runs", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--epochs", type=int, default=20)
    ap.add_argument("--batches", type=int, default=0)
    ap.add_argument("--scale", type=float, default=1.0)
    ap.add_argument("--batch-scale", type=float, default=1.0)
    ap.add_argument("--device", default=None)
    a = ap.parse_args(argv)
    for name in a.models.split(","):
        rows = {}
        for arm in a.arms.split(","):
            try:
                r = run_benchmark(name, arm, a.device, a.runs, a.warmup, a.epochs, a.batches or None,
                                  a.scale, a.batch_scale)
            except Exception as e:  # e.g. a model with host-side control flow under capture
                print(json.dumps({"name": name, "arm": arm, "unavailable": repr(e)[:300]}), flush=True)
                continue
            rows[arm] = r
            print(json.dumps(asdict(r)), flush=True)
        if "flodl" in rows and "torch" in rows:
            f, t = rows["flodl"].median_epoch_ms, rows["torch"].median_epoch_ms
            extra = {}
            if "torch-bf16" in rows:
                extra["speedup_vs_torch_bf16"] = round(rows["torch-bf16"].median_epoch_ms / f, 3)
            if "flodl-graph" in rows:
                extra["graph_speedup_vs_torch_f32"] = round(t / rows["flodl-graph"].median_epoch_ms, 3)
            print(json.dumps({"name": name, "speedup_vs_torch_f32": round(t / f, 3), **extra}),
                  flush=True)


if __name__ == "__main__":
    main()
