"""Kernel micro-benchmarks at the headline model's shapes.

    python -m flodl_b200.bench_kernels [--case NAME|all] [--iters N] [--warmup W]
                                       [--launches K]

Each case builds its inputs once on ``cuda:0`` and times ``iters`` launches
(captured into one CUDA graph, so that the host cost of the binding call does
not hide a short kernel; ``--graph 0`` times eager launches) with CUDA events
after ``warmup`` launches (inputs larger than L2 where the
case is memory-bound), then prints one JSON line per case: microseconds per
launch, the algorithmic FLOPs or bytes, the achieved rate, and its fraction
of the measured peaks in ``MEASURED_PEAKS.json`` (cuBLAS bf16 GEMM burst and
STREAM-style copy bandwidth, measured on this hardware). ``--launches K``
instead runs exactly K launches untimed - the small, bounded workload used
for profiler captures.

Shapes are those of the transformer LM benchmark (64 x 256 tokens, d=512,
8 heads, FFN 2048); the reference's own kernel benchmarks live in
``benchmarks/`` of fab2s/floDl and time libtorch's kernels the same way.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

T, D, H, FF, S, B = 16384, 512, 8, 2048, 256, 64


def _peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def _bf(*s):
    return torch.randn(*s, device="cuda").bfloat16()


def case_gemm(kind):
    from ._ext import cuda_ext
    C = cuda_ext()
    if kind == "gemm_qkv":  # x @ Wqkv^T + b  (bf16 out)
        M, N, K = T, 3 * D, D
        A, Bm = _bf(M, K), _bf(N, K)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        bias = torch.randn(N, device="cuda")
        fn = lambda: C.gemm(A, Bm, out, M, N, K, False, False, bias=bias)
        nbytes = (M * K + N * K + M * N) * 2
    elif kind == "gemm_qkv_nobias":  # the qkv shape without the bias (epilogue cost probe)
        M, N, K = T, 3 * D, D
        A, Bm = _bf(M, K), _bf(N, K)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        fn = lambda: C.gemm(A, Bm, out, M, N, K, False, False)
        nbytes = (M * K + N * K + M * N) * 2
    elif kind == "gemm_fc1_nogelu":  # the fc1 shape with bias only (GELU cost probe)
        M, N, K = T, FF, D
        A, Bm = _bf(M, K), _bf(N, K)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        bias = torch.randn(N, device="cuda")
        fn = lambda: C.gemm(A, Bm, out, M, N, K, False, False, bias=bias)
        nbytes = (M * K + N * K + M * N) * 2
    elif kind == "gemm_fc1_gelu":  # gelu(x W1^T + b1), GELU' kept (two bf16 outputs)
        M, N, K = T, FF, D
        A, Bm = _bf(M, K), _bf(N, K)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        aux = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        bias = torch.randn(N, device="cuda")
        fn = lambda: C.gemm(A, Bm, out, M, N, K, False, False, bias=bias, aux=aux,
                            flags=C.EPI_GELU)
        nbytes = (M * K + N * K + 2 * M * N) * 2
    elif kind == "gemm_fc2_residual":  # x + h W2^T + b2 (f32 residual stream)
        M, N, K = T, D, FF
        A, Bm = _bf(M, K), _bf(N, K)
        out = torch.empty(M, N, device="cuda")
        res = torch.randn(M, N, device="cuda")
        bias = torch.randn(N, device="cuda")
        fn = lambda: C.gemm(A, Bm, out, M, N, K, False, False, bias=bias, residual=res)
        nbytes = (M * K + N * K) * 2 + 2 * M * N * 4
    elif kind == "gemm_dgrad_dgelu":  # (dy W2) * GELU'
        M, N, K = T, FF, D
        A, Bm = _bf(M, K), _bf(K, N)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        g = _bf(M, N)
        fn = lambda: C.gemm(A, Bm, out, M, N, K, False, True, aux=g, flags=C.EPI_DGELU)
        nbytes = (M * K + N * K + 2 * M * N) * 2
    elif kind == "gemm_wgrad":  # dW1 += da^T h (f32, split-K)
        from .ops._common import splitk_for
        M, N, K = FF, D, T
        A, Bm = _bf(K, M), _bf(K, N)
        out = torch.zeros(M, N, device="cuda")
        ks = splitk_for(M, N, K)
        fn = lambda: C.gemm(A, Bm, out, M, N, K, True, True, flags=C.EPI_ACCUMULATE, k_splits=ks)
        nbytes = (M * K + N * K) * 2 + 2 * M * N * 4
    else:
        raise KeyError(kind)
    return fn, 2.0 * M * N * K, nbytes


def case_flash(kind):
    from ._ext import cuda_ext
    C = cuda_ext()
    qkv = _bf(B * S, 3 * D)
    out = torch.empty(B * S, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, H, S, device="cuda")
    sc = 1.0 / math.sqrt(D // H)
    C.flash_attn_fwd(qkv, out, lse, B, S, H, D // H, True, sc)
    # causal attention FLOPs: 4 B H S^2 d / 2 forward, 2.5x that backward
    f_fwd = 4.0 * B * H * S * S * (D // H) / 2
    if kind == "flash_fwd":
        fn = lambda: C.flash_attn_fwd(qkv, out, lse, B, S, H, D // H, True, sc)
        return fn, f_fwd, (B * S * 3 * D + B * S * D) * 2
    dout = _bf(B * S, D)
    dqkv = torch.empty_like(qkv)
    fn = lambda: C.flash_attn_bwd(dout, qkv, out, lse, dqkv, B, S, H, D // H, True, sc)
    return fn, 2.5 * f_fwd, (B * S * 3 * D * 2 + 2 * B * S * D) * 2


def case_flash_bert(kind):
    """BERT-base attention: 32 x 512 tokens, 12 heads of 64, bidirectional,
    key padding (the last 10% of each sequence's keys masked)."""
    from ._ext import cuda_ext
    C = cuda_ext()
    Bb, Sb, Hb, Db = 32, 512, 12, 768
    qkv = _bf(Bb * Sb, 3 * Db)
    out = torch.empty(Bb * Sb, Db, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(Bb, Hb, Sb, device="cuda")
    pad = torch.zeros(Bb, Sb, dtype=torch.bool, device="cuda")
    pad[:, Sb - Sb // 10:] = True
    sc = 1.0 / math.sqrt(Db // Hb)
    C.flash_attn_fwd(qkv, out, lse, Bb, Sb, Hb, Db // Hb, False, sc, pad)
    f_fwd = 4.0 * Bb * Hb * Sb * Sb * (Db // Hb)
    if kind == "flash_fwd_bert":
        fn = lambda: C.flash_attn_fwd(qkv, out, lse, Bb, Sb, Hb, Db // Hb, False, sc, pad)
        return fn, f_fwd, (Bb * Sb * 3 * Db + Bb * Sb * Db) * 2
    dout = _bf(Bb * Sb, Db)
    dqkv = torch.empty_like(qkv)
    fn = lambda: C.flash_attn_bwd(dout, qkv, out, lse, dqkv, Bb, Sb, Hb, Db // Hb, False, sc, pad)
    return fn, 2.5 * f_fwd, (Bb * Sb * 3 * Db * 2 + 2 * Bb * Sb * Db) * 2


def case_ln(kind):
    from ._ext import cuda_ext
    C = cuda_ext()
    x = torch.randn(T, D, device="cuda")
    w = torch.randn(D, device="cuda")
    b = torch.randn(D, device="cuda")
    y16 = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
    mean = torch.empty(T, device="cuda")
    rstd = torch.empty(T, device="cuda")
    C.ln_fwd(x, w, b, y16, None, mean, rstd, 1e-5)
    if kind == "ln_fwd":
        fn = lambda: C.ln_fwd(x, w, b, y16, None, mean, rstd, 1e-5)
        return fn, 0.0, T * D * (4 + 2) + T * 8
    dy = _bf(T, D)
    dres = torch.randn(T, D, device="cuda")
    dx = torch.empty(T, D, device="cuda")
    dx16 = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
    dw = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    dbias = torch.zeros(D, device="cuda")
    fn = lambda: C.ln_bwd(dy, x, mean, rstd, w, dres, dx, dx16, dw, db, dbias)
    return fn, 0.0, T * D * (2 + 4 + 4 + 4 + 2)


def case_adamw(_):
    from ._ext import cuda_ext
    C = cuda_ext()
    n = 19 * (1 << 20)
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    sh = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    lr = torch.full((), 3e-4, device="cuda")
    step = torch.ones((), device="cuda")
    fn = lambda: C.adamw(p, g, m, v, sh, lr, step, None, 0.9, 0.999, 1e-8, 0.1, True, False)
    return fn, 0.0, n * (4 * 4 + 3 * 4 + 2)


def case_sgd(_):
    from ._ext import cuda_ext
    C = cuda_ext()
    n = 19 * (1 << 20)
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    buf = torch.zeros(n, device="cuda")
    sh = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    lr = torch.full((), 0.1, device="cuda")
    first = torch.zeros((), device="cuda")
    fn = lambda: C.sgd(p, g, buf, sh, lr, None, first, 0.9, 0.0, 0.0, False, False)
    return fn, 0.0, n * (3 * 4 + 2 * 4 + 2)


def case_softmax_ce(_):
    # the LM head's loss: 16384 rows x 256 byte classes, bf16 logits, dlogits out
    from ._ext import cuda_ext
    C = cuda_ext()
    V = 256
    logits = _bf(T, V)
    tgt = torch.randint(0, V, (T,), device="cuda")
    loss = torch.zeros((), device="cuda")
    inv = torch.zeros((), device="cuda")
    dl = torch.empty(T, V, device="cuda", dtype=torch.bfloat16)
    fn = lambda: C.softmax_ce(logits, tgt, loss, inv, dl, -100, 0.0)
    return fn, 0.0, T * V * 2 * 2 + T * 8


def case_embed(kind):
    # token + position embedding of the LM batch (f32 residual stream and bf16 copy)
    from ._ext import cuda_ext
    C = cuda_ext()
    V = 256
    ids = torch.randint(0, V, (B, S), device="cuda")
    tok = torch.randn(V, D, device="cuda")
    pos = torch.randn(S, D, device="cuda")
    out = torch.empty(T, D, device="cuda")
    out16 = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
    if kind == "embed_fwd":
        fn = lambda: C.embed_fwd(ids, tok, pos, None, None, out, out16, S)
        return fn, 0.0, T * D * (4 + 2) + T * 8
    dy = torch.randn(T, D, device="cuda")
    dtok = torch.zeros(V, D, device="cuda")
    fn = lambda: C.embed_bwd_atomic(ids, dy, dtok)
    return fn, 0.0, T * D * 4 + T * 8


# ResNet-20 stage-1 activation of the config-2 batch: 128 x 32 x 32 x 16 (NHWC bf16)
RN, RH, RC = 128, 32, 16


def case_conv(kind):
    from ._ext import cuda_ext
    C = cuda_ext()
    x = _bf(RN, RH, RH, RC)
    M = RN * RH * RH
    if kind == "col2im_bn":  # col2im (+ add, * mask) with the batch-norm backward sums
        dcols = _bf(M, 9 * RC)
        dz = torch.empty_like(x)
        add, mask, y = _bf(RN, RH, RH, RC), _bf(RN, RH, RH, RC), _bf(M, RC)
        mean = torch.zeros(RC, device="cuda")
        rstd = torch.ones(RC, device="cuda")
        ws = torch.zeros(2 * RC + 1, device="cuda")
        sums = torch.zeros(2 * RC, device="cuda")
        dg, db = torch.zeros(RC, device="cuda"), torch.zeros(RC, device="cuda")
        fn = lambda: C.col2im_bn(dcols, dz, 3, 1, 1, add, mask, y, mean, rstd, dg, db, sums, ws)
        return fn, 0.0, M * 9 * RC * 2 + 4 * M * RC * 2
    if kind in ("im2col", "col2im"):
        cols = torch.empty(M, 9 * RC, device="cuda", dtype=torch.bfloat16)
        if kind == "im2col":
            fn = lambda: C.im2col(x, cols, 3, 1, 1)
            return fn, 0.0, M * RC * 2 + M * 9 * RC * 2
        dcols = _bf(M, 9 * RC)
        dx = torch.empty_like(x)
        fn = lambda: C.col2im(dcols, dx, 3, 1, 1, None, None)
        return fn, 0.0, M * 9 * RC * 2 + M * RC * 2
    mean = torch.empty(RC, device="cuda")
    rstd = torch.empty(RC, device="cuda")
    rm = torch.zeros(RC, device="cuda")
    rv = torch.ones(RC, device="cuda")
    ws = torch.zeros(2 * RC + 1, device="cuda")
    gamma = torch.ones(RC, device="cuda")
    beta = torch.zeros(RC, device="cuda")
    C.bn_stats(x, mean, rstd, rm, rv, ws, 1e-5, 0.1)
    if kind == "bn_stats":
        fn = lambda: C.bn_stats(x, mean, rstd, rm, rv, ws, 1e-5, 0.1)
        return fn, 0.0, M * RC * 2
    if kind == "bn_apply":
        y = torch.empty_like(x)
        ident = _bf(RN, RH, RH, RC)
        fn = lambda: C.bn_apply(x, mean, rstd, gamma, beta, ident, True, y)
        return fn, 0.0, 3 * M * RC * 2
    dy = _bf(RN, RH, RH, RC)
    ymask = _bf(RN, RH, RH, RC)
    dg = torch.zeros(RC, device="cuda")
    db = torch.zeros(RC, device="cuda")
    sums = torch.zeros(2 * RC, device="cuda")
    dx = torch.empty_like(x)
    fn = lambda: C.bn_bwd(dy, ymask, x, mean, rstd, gamma, dg, db, sums, ws, dx, None)
    return fn, 0.0, 2 * (3 * M * RC * 2) + M * RC * 2


def case_norms(kind):
    """RMSNorm (BERT-width rows), GroupNorm and max pooling (ResNet-like
    activations), forward + backward per launch pair."""
    from ._ext import cuda_ext
    C = cuda_ext()
    if kind == "rmsnorm":
        rows, Cd = T, 768
        x = torch.randn(rows, Cd, device="cuda")
        w = torch.rand(Cd, device="cuda") + 0.5
        y, dx = torch.empty_like(x), torch.empty_like(x)
        rstd = torch.empty(rows, device="cuda")
        dy = torch.randn_like(x)
        dw = torch.zeros(Cd, device="cuda")

        def fn():
            C.rms_fwd(x, w, y, rstd, 1e-5)
            C.rms_bwd(dy, x, w, rstd, dx, dw)
        return fn, 0.0, (2 + 3) * rows * Cd * 4  # fwd: x, y; bwd: dy, x, dx
    if kind == "groupnorm":
        N, Cc, HW, G = 128, 64, 32 * 32, 32
        x = torch.randn(N, Cc, HW, device="cuda")
        w, b = torch.rand(Cc, device="cuda") + 0.5, torch.randn(Cc, device="cuda")
        y, dx = torch.empty_like(x), torch.empty_like(x)
        mean, rstd = torch.empty(N * G, device="cuda"), torch.empty(N * G, device="cuda")
        dy = torch.randn_like(x)
        dg, db = torch.zeros(Cc, device="cuda"), torch.zeros(Cc, device="cuda")

        def fn():
            C.gn_fwd(x, w, b, y, mean, rstd, G, 1e-5)
            C.gn_bwd(dy, x, w, mean, rstd, dx, dg, db, G)
        return fn, 0.0, (2 + 3) * x.numel() * 4
    N, Cc, H = 128, 64, 64  # max pooling 2x2 / 2
    x = torch.randn(N, Cc, H, H, device="cuda")
    y = torch.empty(N, Cc, H // 2, H // 2, device="cuda")
    idx = torch.empty(y.shape, device="cuda", dtype=torch.int32)
    dx = torch.zeros_like(x)
    dy = torch.randn_like(y)

    def fn():
        C.maxpool_fwd(x, y, idx, 2, 2, 2, 2, 0, 0, 1, 1)
        C.maxpool_bwd(dy, idx, dx)
    return fn, 0.0, x.numel() * 4 + y.numel() * 8 + y.numel() * 8 + x.numel() * 4


CASES = {
    "gemm_qkv": case_gemm, "gemm_fc1_gelu": case_gemm, "gemm_fc2_residual": case_gemm,
    "gemm_dgrad_dgelu": case_gemm, "gemm_wgrad": case_gemm, "gemm_qkv_nobias": case_gemm,
    "gemm_fc1_nogelu": case_gemm,
    "flash_fwd": case_flash, "flash_bwd": case_flash,
    "flash_fwd_bert": case_flash_bert, "flash_bwd_bert": case_flash_bert,
    "ln_fwd": case_ln, "ln_bwd": case_ln, "adamw": case_adamw, "sgd": case_sgd,
    "softmax_ce": case_softmax_ce, "embed_fwd": case_embed, "embed_bwd": case_embed,
    "im2col": case_conv, "col2im": case_conv, "bn_stats": case_conv, "bn_apply": case_conv,
    "bn_bwd": case_conv, "col2im_bn": case_conv,
    "rmsnorm": case_norms, "groupnorm": case_norms, "maxpool": case_norms,
}


def run(name, iters, warmup, launches, graph=True):
    fn, flops, nbytes = CASES[name](name)
    if launches:
        for _ in range(launches):
            fn()
        torch.cuda.synchronize()
        return {"case": name, "launches": launches}
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        # `iters` launches captured into one CUDA graph: device time without
        # the host cost of the binding calls (which exceeds short kernels)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
    else:
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / iters
    tf_peak, bw_peak, src = _peaks()
    rec = {"case": name, "us": round(us, 2), "timing": "graph" if graph else "eager"}
    if flops:
        tf = flops / us / 1e6
        rec.update(tflops=round(tf, 1), frac_of_bf16_peak=round(tf / tf_peak, 3))
    gbs = nbytes / us / 1e3
    rec.update(gbs=round(gbs, 1), frac_of_hbm=round(gbs / bw_peak, 3), peaks=src)
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--launches", type=int, default=0)
    ap.add_argument("--graph", type=int, default=1,
                    help="time a CUDA graph of the launches (1) or eager launches (0)")
    a = ap.parse_args()
    names = list(CASES) if a.case == "all" else a.case.split(",")
    for n in names:
        print(json.dumps(run(n, a.iters, a.warmup, a.launches, bool(a.graph))), flush=True)


if __name__ == "__main__":
    main()
