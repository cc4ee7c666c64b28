"""Collective benchmarks on one NVLink/NVSwitch node.

Launch one rank per GPU (``torchrun --nproc-per-node N --master-addr 127.0.0.1
-m flodl_b200.parallel.bench_collectives --mode ...``); rank 0 prints JSON
lines. All times are CUDA-event device times, max over ranks.

Modes:

* ``sweep``     all-reduce (sum) of fp32 and bf16 buffers from 4 KiB to 1 GiB:
                the peer-memory kernel (fp32, two-shot and one-shot) and NCCL
                (fp32, bf16); algorithmic and bus bandwidth (2 (n-1)/n x bytes
                / time).
* ``fused``     the fused gradient all-reduce + AdamW kernel on a parameter
                arena the size of the LM benchmark (or ``--numel``), reported
                against its NVLink roofline. Out of each GPU go the peers' reads
                of their shards of its f32 gradients ((n-1)/n x 4 B per
                element) and its shard's f32 weights and bf16 shadows written
                into every peer ((n-1)/n x 6 B); both use the same direction of
                the GPU's NVLink port, so the target time is (n-1)/n x 10 B x
                elements over the measured 770 GB/s per-direction peer copy
                bandwidth.
* ``averaging`` cluster parameter averaging with uneven work: ResNet-20,
                rank r runs 4 + r local SGD steps per round on its own batch,
                then the parameters are averaged weighted by the steps each
                rank did (the reference's realized-work mass), through the fused
                weighted-average kernel (``--engine peer``) or NCCL
                (``--engine nccl``: scale, all-reduce, divide).
* ``avgkernel`` the weighted-average kernel alone against its NVLink roofline.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured peer copy bandwidth per direction (B200 NVLink 5)


def _init():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    return rank, world, dev


def _time(fn, iters, warmup, world):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())  # ms


def _time_graph(fn, iters, warmup, world):
    """Device time per call of `fn` with host launch cost removed: `iters`
    calls are captured into one CUDA graph and the replay is timed (max over
    ranks). NCCL and the peer kernels both capture; the graph is released
    before returning (a graph holding NCCL work must not outlive the group)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())  # ms


def sweep(rank, world, dev, args):
    """Two-shot and one-shot peer all-reduce against NCCL. One-shot reads
    every peer's whole buffer (world x the bytes of two-shot) and is timed up
    to ``--oneshot-max-log2``."""
    from .peer import PeerComm
    max_bytes = 1 << args.max_log2
    comm = PeerComm(max_bytes // 4, dev, with_shadow=False, timeout_s=10.0)
    timer = _time_graph if args.graph else _time
    buf = torch.empty(max_bytes // 4, device=dev)
    buf16 = torch.empty(max_bytes // 2, device=dev, dtype=torch.bfloat16)
    nb = args.min_log2
    while nb <= args.max_log2:
        nbytes = 1 << nb
        iters = 50 if nbytes <= (64 << 20) else 10
        n32 = max(nbytes // 4, 4)
        comm.grad[:n32].fill_(1.0)
        t_peer = timer(lambda: comm.all_reduce_(n32, average=False, slot=0), iters, 3, world)
        t_one = None
        if nb <= args.oneshot_max_log2:
            t_one = timer(lambda: comm.all_reduce_(n32, average=False, slot=1, oneshot=True),
                          iters, 3, world)
        comm.check()
        t_nccl = timer(lambda: dist.all_reduce(buf[:n32]), iters, 3, world)
        n16 = max(nbytes // 2, 8)
        t_nccl16 = timer(lambda: dist.all_reduce(buf16[:n16]), iters, 3, world)
        if rank == 0:
            f = 2.0 * (world - 1) / world
            rec = {"mode": "sweep", "n_gpus": world, "bytes": nbytes,
                   "timing": "cuda-graph replay" if args.graph else "eager launches"}
            for name, t in (("peer_f32", t_peer), ("peer_oneshot_f32", t_one),
                            ("nccl_f32", t_nccl), ("nccl_bf16", t_nccl16)):
                if t is None:
                    continue
                rec[name] = {"us": round(t * 1e3, 2), "algbw_gbs": round(nbytes / t / 1e6, 2),
                             "busbw_gbs": round(f * nbytes / t / 1e6, 2)}
            best = min(t for t in (t_peer, t_one) if t is not None)
            rec["peer_best_over_nccl"] = round(t_nccl / best, 3)
            print(json.dumps(rec), flush=True)
        nb += args.step_log2
    comm.close()


def fused(rank, world, dev, args):
    from .peer import PeerComm
    n = (args.numel + 63) // 64 * 64
    comm = PeerComm(n, dev, timeout_s=10.0)
    C = comm.C
    comm.data[:n].normal_()
    comm.grad[:n].normal_()
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    lr = torch.full((), 1e-4, device=dev)
    step = torch.ones((), device=dev)
    buckets = max(1, args.buckets)
    per = (n // buckets + 63) // 64 * 64

    def run():
        for i in range(buckets):
            s0 = i * per
            s1 = min(n, s0 + per)
            if s0 >= s1:
                break
            comm.launch(C.FUSED_AR_ADAMW, bucket=i, start=s0, end=s1, blocks=args.blocks,
                        m=m, v=v, lr=lr, step=step, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.1,
                        oneshot=int(args.oneshot))

    t = _time(run, 20, 3, world)
    comm.check()
    # bytes leaving each GPU (and, by symmetry, arriving): the peers read
    # their shards of this rank's f32 gradients ((n-1)/n x 4 B per element)
    # and this rank writes its shard's f32 weights and bf16 shadow into every
    # peer ((n-1)/n x 6 B); both share the link direction out of this GPU
    frac = (world - 1) / world
    link_bytes = frac * (4 + 6) * n
    target_ms = link_bytes / (LINK_GBS * 1e9) * 1e3
    if rank == 0:
        print(json.dumps({"mode": "fused_allreduce_adamw", "n_gpus": world, "numel": n,
                          "buckets": buckets, "oneshot": bool(args.oneshot),
                          "us": round(t * 1e3, 2),
                          "nvlink_roofline_us": round(target_ms * 1e3, 2),
                          "frac_of_roofline": round(target_ms / t, 3) if world > 1 else None,
                          "link_gbs_assumed": LINK_GBS}), flush=True)
    comm.close()


def averaging(rank, world, dev, args):
    from ..models import ResNet20
    from ..optim import SGD
    from ..utils.arena import ParamArena
    from .config import AverageBackend
    torch.manual_seed(0)
    model = ResNet20(device=dev)
    params = list(model.parameters())
    avg = None
    opt = SGD(params, lr=0.1, momentum=0.9, weight_decay=1e-4)
    if args.engine == "peer" and world > 1:
        from .trainer import _Averager
        # parameters and BatchNorm statistics averaged by one fused kernel
        avg = _Averager(model, opt, AverageBackend.NCCL, rank, world, dev)
        arena = avg.fused[1]
    else:
        arena = ParamArena(params)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(128, 3, 32, 32, device=dev, generator=g)
    y = torch.randint(0, 10, (128,), device=dev, generator=g)
    local_steps = 4 + rank
    steps = [local_steps]
    if world > 1:
        all_steps = [None] * world
        dist.all_gather_object(all_steps, local_steps)
        steps = all_steps
    bufs = [b for b in model.buffers() if b.dtype == torch.float32]

    def round_():
        for _ in range(local_steps):
            loss = model.loss(x, y)
            loss.backward()
            opt.step()
            opt.zero_grad()
        if world == 1:
            return
        mass = float(local_steps)
        if avg is not None:
            avg.average(local_steps)
        else:
            arena.data.mul_(mass / float(sum(steps)))
            dist.all_reduce(arena.data)
            arena.refresh_shadow()
            for b in bufs:  # batch-norm running statistics: mean over the ranks that moved
                b.mul_(1.0 / world)
                dist.all_reduce(b)

    t = _time(round_, args.rounds, 2, world)
    samples = 128 * sum(steps)
    if rank == 0:
        print(json.dumps({"mode": "averaging", "engine": args.engine if world > 1 else "none",
                          "n_gpus": world, "model": "resnet20", "batch_per_step": 128,
                          "local_steps_per_rank": steps, "round_ms": round(t, 3),
                          "samples_per_s": round(samples / (t / 1e3), 1),
                          "note": "device time per round (local steps + weighted average), max over ranks"}),
              flush=True)
    if avg is not None:
        avg.close()


def avgkernel(rank, world, dev, args):
    """The weighted-average kernel alone (parameters + an f32 buffer tail,
    divergence partials on) against its NVLink roofline: rank r reads shard r
    of every peer ((n-1)/n x 4 bytes per element) and writes the average and
    its bf16 shadow into every peer ((n-1)/n x 6 bytes per element)."""
    from .peer import PeerComm
    n = (args.numel + 63) // 64 * 64
    nbuf = 4096
    comm = PeerComm(n + nbuf, dev, timeout_s=10.0)
    comm.data.normal_()
    div = torch.zeros(2, device=dev)

    def run():
        comm.weighted_average_(n + nbuf, float(1 + rank), slot=0, div=div, buf_start=n)

    t = _time(run, 20, 3, world)
    comm.check()
    frac = (world - 1) / world
    # out of each GPU: the peers' reads of their shards of this rank's data
    # (4 B per element) plus this rank's average and shadow written into
    # every peer (6 B per element), each (n-1)/n of the elements
    target_ms = frac * 10 * (n + nbuf) / (LINK_GBS * 1e9) * 1e3
    if rank == 0:
        print(json.dumps({"mode": "weighted_average_kernel", "n_gpus": world,
                          "numel": n, "buffer_numel": nbuf, "us": round(t * 1e3, 2),
                          "nvlink_roofline_us": round(target_ms * 1e3, 2),
                          "frac_of_roofline": round(target_ms / t, 3) if world > 1 else None,
                          "link_gbs_assumed": LINK_GBS}), flush=True)
    comm.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", default="sweep", choices=["sweep", "fused", "averaging", "avgkernel"])
    ap.add_argument("--max-log2", type=int, default=30)
    ap.add_argument("--min-log2", type=int, default=12)
    ap.add_argument("--step-log2", type=int, default=2)
    ap.add_argument("--oneshot-max-log2", type=int, default=24)
    ap.add_argument("--oneshot", action="store_true")
    ap.add_argument("--numel", type=int, default=19_000_000)
    ap.add_argument("--buckets", type=int, default=4)
    ap.add_argument("--blocks", type=int, default=0)
    ap.add_argument("--engine", default="peer", choices=["peer", "nccl"])
    ap.add_argument("--rounds", type=int, default=10)
    ap.add_argument("--graph", type=int, default=1,
                    help="sweep: time CUDA-graph replays (device latency, no host launch cost)")
    args = ap.parse_args()
    rank, world, dev = _init()
    {"sweep": sweep, "fused": fused, "averaging": averaging,
     "avgkernel": avgkernel}[args.mode](rank, world, dev, args)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
