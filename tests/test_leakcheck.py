"""Leak checks: resident memory stays bounded over many iterations of the
host-side paths that allocate per call (reference: the `*leakcheck` tests run
serially in CI)."""
import gc
import os

import torch

from flodl_b200.graph import FlowBuilder
from flodl_b200.nn import GELU, LayerNorm, Linear, mse_loss
from flodl_b200.optim import Adam


def _rss_mb() -> float:
    with open(f"/proc/{os.getpid()}/statm") as f:
        return int(f.read().split()[1]) * os.sysconf("SC_PAGE_SIZE") / 2 ** 20


def _steady(fn, warm=30, iters=300, slack_mb=24.0):
    for _ in range(warm):
        fn()
    gc.collect()
    base = _rss_mb()
    for _ in range(iters):
        fn()
    gc.collect()
    grown = _rss_mb() - base
    assert grown < slack_mb, f"resident memory grew {grown:.1f} MB over {iters} iterations"


def test_leakcheck_graph_training_step():
    g = FlowBuilder.from_(Linear(64, 128)).through(GELU()).through(LayerNorm(128)).through(Linear(128, 8)).build()
    opt = Adam(g.parameters(), lr=1e-3)
    x, y = torch.randn(32, 64), torch.randn(32, 8)

    def step():
        loss = mse_loss(g(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad()
    _steady(step)


def test_leakcheck_checkpoint_save_load(tmp_path):
    from flodl_b200.nn.checkpoint import load_checkpoint, save_checkpoint
    g = FlowBuilder.from_(Linear(64, 64)).build()
    p = str(tmp_path / "m.fdl")

    def roundtrip():
        save_checkpoint(p, g.graph_named_parameters(), (), g.structural_hash())
        load_checkpoint(p, g.graph_named_parameters(), (), g.structural_hash())
    _steady(roundtrip, iters=200)


def test_leakcheck_wire_frames():
    from flodl_b200._ext import native
    N = native()
    key = b"k" * 16
    payload = os.urandom(1 << 16)

    def frame():
        N.decode_frame(N.encode_frame(0x1234, 1, 7, payload, key), key, 1 << 20)
    _steady(frame, iters=2000)
