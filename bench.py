#!/usr/bin/env python
"""Headline benchmark: transformer-LM DDP training throughput on B200.

Config: decoder-only LM, 6 layers, d_model 512,
8 heads, MLP 2048 GELU, pre-LayerNorm, vocab 256 (uniform random byte tokens),
seq 256, batch 64 per GPU, bf16 compute / f32 master weights, AdamW lr 3e-4
wd 0.1. Weak scaling: global batch = 64 x N.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flodl|reference|torch]
                    [--model lm|bert]

``--model bert`` runs BASELINE config 4 instead (BERT-base MLM, seq 512,
batch 32 per GPU, 15% of positions masked, AdamW).

N > 1 runs under torchrun (one rank per GPU, NCCL bootstrap). Each timed
window is exactly K steps bracketed by barrier + synchronize, timed with CUDA
events on the launching stream, max over ranks; ``--windows`` (5) such windows
run back to back and the median is reported with the spread; rank 0 prints
one JSON line.

``value`` is the device-timed whole-step throughput of the captured step (CUDA
graph replay: forward, backward, gradient all-reduce, AdamW). ``e2e`` runs the
public training API (``flodl_b200.train.StepRunner``) with the step's inputs
copied from pinned host memory and the loss read back every step.

``--impl reference`` runs the unmodified reference (fab2s/floDl) if it is
installed under baseline/_ref; it is a Rust/cargo workspace that this image
cannot build, so the arm reports ``unavailable``. ``--impl torch`` is an extra
proxy arm: the same model written with stock PyTorch modules (cuBLAS, SDPA
flash attention, fused AdamW, NCCL DDP) — the library calls the reference
itself makes through libtorch.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "DDP samples/s & tok/s, 1/2/4/8 B200, max-over-ranks vs ref NCCL build"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="flodl", choices=["flodl", "reference", "torch"])
    ap.add_argument("--engine", default="auto", choices=["auto", "nccl", "peer"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--windows", type=int, default=5,
                    help="timed windows of --steps steps each; the median window is reported")
    ap.add_argument("--model", default="lm", choices=["lm", "bert", "resnet20"],
                    help="lm = BASELINE config 3 (the headline); bert = config 4; resnet20 = config 2")
    return ap.parse_args()


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_arm(args):
    ref = os.path.join(ROOT, "baseline", "_ref")
    msg = ("reference fab2s/floDl is a Rust/cargo workspace (no setup.py/pyproject); "
           "pip install of the reference source tree fails and no Rust toolchain (cargo/rustc) "
           "exists on this image or on the GPU box (probed)")
    if not os.path.isdir(ref) or not os.listdir(ref):
        print(json.dumps({"impl": "reference", "unavailable": msg}))
        return 0
    print(json.dumps({"impl": "reference", "unavailable": msg + " (baseline/_ref holds no runnable build)"}))
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        # the reference arm never imports this package (nor maps its .so files)
        return reference_arm(args)
    from flodl_b200.utils.crash import install_crash_handler
    install_crash_handler()
    import torch
    import torch.distributed as dist

    from flodl_b200.parallel.ddp import init_from_env

    rank, world, local = init_from_env("nccl", timeout_s=300)
    if world != args.gpus and args.gpus > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    torch.manual_seed(1234)
    torch.backends.cuda.matmul.allow_tf32 = False

    from flodl_b200.bench_support import MODELS
    spec = MODELS[args.model]
    B_PER_GPU, SEQ = spec.batch, spec.seq
    UNIT = "samples/s" if SEQ == 1 else "tok/s"  # image models: one sample per "token"
    if args.impl == "torch":
        step, state = spec.torch(dev, world)
        engine = "nccl(torch DDP)"
        launches_fn = None
    else:
        engine = args.engine
        if engine == "auto":
            engine = "peer" if world > 1 else "none"
        step, state = spec.flodl(dev, world, engine)
        from flodl_b200._ext import cuda_ext
        launches_fn = cuda_ext().launch_count

    # warm-up (eager, on a side stream so every buffer the step creates - arenas,
    # gradients, workspaces - belongs to a non-legacy stream before capture)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()

    graph = None
    # stock torch DDP cannot be captured into a CUDA graph (its reducer
    # issues host-side work during backward): the torch arm runs eager at N > 1
    if not args.no_graph and not (args.impl == "torch" and world > 1):
        graph = torch.cuda.CUDAGraph()
        c0 = launches_fn() if launches_fn else 0
        with torch.cuda.graph(graph):
            static_loss = step()
        per_step_launches = (launches_fn() - c0) if launches_fn else None
        run = graph.replay
        for _ in range(2):
            run()
    else:
        c0 = launches_fn() if launches_fn else 0
        step()
        per_step_launches = (launches_fn() - c0) if launches_fn else None
        run = step
    torch.cuda.synchronize()

    # ---------------------------------------------------------------- timed (device)
    # `--windows` windows of exactly K steps, each bracketed by barrier +
    # synchronize and timed with CUDA events on the launching stream; a
    # window's time is the max over ranks; the reported value is the median
    # window, with the spread of all windows alongside.
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    windows = []
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    for _ in range(max(1, args.windows)):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            run()
        e1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        windows.append(float(t.item()))
    clocks = sampler.stop()
    ms = statistics.median(windows)
    spread = {"windows": len(windows), "ms_per_step_min": min(windows),
              "ms_per_step_max": max(windows),
              "rel_spread": (max(windows) - min(windows)) / ms if ms > 0 else None}

    # ---------------------------------------------------------------- e2e (public API)
    e2e = None
    if args.impl == "flodl":
        from flodl_b200.train import StepRunner
        runner = StepRunner(step, state["inputs"], graph, static_loss if graph else None)
        host_in = state["host_inputs"]()
        n_e2e = args.e2e_steps or args.steps
        runner.step(*host_in)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        for _ in range(n_e2e):
            # H2D inputs, replay, D2H loss (each step's loss is read on the
            # host while the next step runs)
            runner.step_pipelined(*host_in)
        runner.flush()
        torch.cuda.synchronize()
        e2e_ms = (time.perf_counter() - w0) * 1e3 / n_e2e
        te = torch.tensor([e2e_ms], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item())
        e2e = {"value": world * B_PER_GPU * SEQ / (e2e_ms / 1e3), "unit": UNIT,
               "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host_in),
               "d2h_bytes_per_step": 4,
               "api": "flodl_b200.train.StepRunner.step_pipelined (loss of step i read on the host during step i+1)"}

    tok_s = world * B_PER_GPU * SEQ / (ms / 1e3)
    if rank == 0:
        out = {
            "metric": METRIC, "value": tok_s, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "samples_per_s": world * B_PER_GPU / (ms / 1e3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (uniform random tokens), random-init weights",
            "config": {"model": spec.desc, "global_batch": B_PER_GPU * world, "seq_len": SEQ,
                       "parallelism": f"dp{world}", "optimizer": spec.optimizer,
                       "grad_allreduce": engine, "cuda_graph": graph is not None,
                       "l2": "inputs larger than L2: ~2 GB of activations per step per GPU"},
            "impl": args.impl,
            "clocks": clocks,
            "timing": spread,
            "e2e": e2e,
            "gpu_launches": (per_step_launches * args.steps) if per_step_launches is not None else None,
        }
        print(json.dumps(out), flush=True)
    # every reference to a CUDA graph that holds NCCL work must be gone before
    # the process group is destroyed, or the exit waits on it forever
    runner = None
    run = None
    static_loss = None
    graph = None
    ddp = state.get("ddp") if isinstance(state, dict) else None
    state = None
    step = None
    import gc
    gc.collect()
    torch.cuda.synchronize()
    if ddp is not None and hasattr(ddp, "close"):
        ddp.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
