"""Managed (``Trainer``) and cooperative (``into_worker``) training tiers.

Reference: ``Trainer::builder(model_factory, optim_factory, train_fn)`` ->
``DdpBuilder`` -> ``.run()`` -> ``DdpHandle::join()`` -> ``TrainedState``
(flodl/src/distributed/ddp.rs:408-560, ddp_run/*). With two or more GPUs the
trainer auto-promotes to one process per GPU; each rank owns a model and
optimizer replica and trains on its shard of the data. Averaging follows the
``ElCheMode``:

* Sync:    every rank steps its optimizer, then parameters (work-weighted)
           and f32 buffers (mean over the ranks that moved) are averaged
           every window of one step.
* Cadence: rank r runs ``batch_counts[r]`` steps per window (ElChe balances
           the counts from measured ms/batch and the averaging overhead), then
           the work-weighted average ``sum_r n_r^gamma W_r / sum n^gamma``.
* Async (CPU backend): each rank blends with the current consensus
           (EASGD) instead of overwriting.

Device averaging runs the fused peer-memory weighted-average kernel on CUDA
(the count exchange rides its signal words); on CPU ranks (gloo) it is a
weighted ``all_reduce``. The CPU backend goes through the signed-frame CPU
reducer hosted by rank 0. Divergence ||pre-post||/||post|| feeds the
convergence guard, which can nudge the ElChe anchor down. Outer optimizers
(SlowMo / DiLoCo) apply to each consensus.

``model_factory(device)``, ``optim_factory(params)`` and ``train_fn(model,
batch) -> loss`` must be picklable (module-level) for multi-process runs.
"""
from __future__ import annotations

import datetime
import os
import queue
import socket
import time
import traceback
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional

import torch
import torch.distributed as dist

from ..data.loader import DataLoader
from ..data.sampler import DistributedSampler
from ..utils import log
from .config import AverageBackend, ApplyPolicy, ElCheConfig, ElCheMode, TrainerConfig
from .convergence import GrowthGuard, LevelGuard, NoGuard, Verdict, divergence, realized_mass
from .outer import OuterAvg, OuterStepper, easgd_blend


@dataclass
class TrainedState:
    params: List = field(default_factory=list)       # [(name, cpu tensor)]
    buffers: List = field(default_factory=list)
    losses: List[float] = field(default_factory=list)  # per-epoch mean loss (rank 0)
    world: int = 1
    mode: str = ""
    syncs: int = 0
    batch_counts: List[List[int]] = field(default_factory=list)
    divergence: List[float] = field(default_factory=list)
    start_epoch: int = 0
    meta_nudges: List[float] = field(default_factory=list)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _flat(params) -> torch.Tensor:
    return torch.cat([p.detach().reshape(-1).float() for p in params])


def _unflat_(params, flat: torch.Tensor) -> None:
    off = 0
    with torch.no_grad():
        for p in params:
            n = p.numel()
            p.copy_(flat[off:off + n].view_as(p).to(p.dtype))
            off += n


class _Averager:
    """Weighted parameter (and f32 buffer) average across ranks for one replica.

    Parameters are averaged with the work mass n^gamma of each rank; f32
    buffers (BatchNorm running statistics and the like) with equal weight over
    the ranks that did any work, as the reference's buffer round does
    (flodl/src/distributed/ddp_run/worker/sync.rs:214-226). When no rank did
    any work nothing changes. On CUDA both rounds are one fused peer-memory
    kernel whose divergence partials come back with the result; on CPU ranks
    they are gloo all-reduces (or the CPU reducer's rounds). ``easgd_alpha``
    blends the consensus into the local replica, ``(1 - a) local + a center``
    (the CpuAsync load, worker/sync.rs:451), instead of overwriting it."""

    def __init__(self, model, opt, backend: AverageBackend, rank: int, world: int, device,
                 cpu_client=None, gamma: float = 1.0, easgd_alpha: Optional[float] = None):
        self.model, self.opt = model, opt
        self.backend, self.rank, self.world = backend, rank, world
        self.device = device
        self.params = [p for p in model.parameters()]
        self.buffers = [b for b in model.buffers() if b.dtype == torch.float32]
        self.cpu = cpu_client
        self.gamma = gamma
        self.alpha = easgd_alpha
        self.fused = None
        self.round = 0
        if backend == AverageBackend.NCCL and device.type == "cuda" and world > 1:
            from ..utils.arena import ParamArena
            from .peer import PeerComm

            nparam = sum((p.numel() + 63) // 64 * 64 for p in self.params)
            self.nbuf = sum(b.numel() for b in self.buffers)
            comm = PeerComm(nparam + (self.nbuf + 63) // 64 * 64, device)
            arena = ParamArena(self.params, alloc=comm.data_alloc, grad_alloc=comm.grad_alloc,
                               with_shadow=False)
            arena.shadow = comm.shadow[:arena.numel]
            arena.rebind()
            arena.refresh_shadow()
            self.fused = (comm, arena)
            self.buf_start = arena.numel
            self.buf_view = comm.data[self.buf_start:self.buf_start + self.nbuf]
            self.div = torch.zeros(2, dtype=torch.float32, device=device)
            for g in opt.groups:
                if all(any(q is p for q in arena.params) for p in g.params) and len(opt.groups) == 1:
                    g.arena = arena

    def flat(self) -> torch.Tensor:
        if self.fused is not None:
            return self.fused[1].data.clone()
        return _flat(self.params)

    def _buffers_flat(self) -> Optional[torch.Tensor]:
        if not self.buffers:
            return None
        return torch.cat([b.detach().reshape(-1) for b in self.buffers])

    def _load_buffers(self, flat: torch.Tensor) -> None:
        off = 0
        with torch.no_grad():
            for b in self.buffers:
                n = b.numel()
                b.copy_(flat[off:off + n].view_as(b))
                off += n

    def average(self, batches: int) -> float:
        """Average with this rank's work; returns ||pre - post|| / ||post||."""
        mass = realized_mass(batches, self.gamma)
        mover = 1.0 if batches > 0 else 0.0
        self.round += 1
        if self.world == 1:
            return 0.0
        if self.fused is not None:
            comm, arena = self.fused
            n = arena.numel
            if self.buffers:
                with torch.no_grad():
                    self.buf_view.copy_(self._buffers_flat())
                n = self.buf_start + self.nbuf
            self.div.zero_()
            comm.weighted_average_(n, mass, slot=0, div=self.div, mover=mover,
                                   buf_start=self.buf_start if self.buffers else -1)
            if self.buffers:
                self._load_buffers(self.buf_view)
            d2, p2 = self.div.tolist()  # synchronises
            comm.check()
            return (d2 ** 0.5) / max(p2 ** 0.5, 1e-12)
        pre = _flat(self.params)
        bpre = self._buffers_flat()
        if self.backend == AverageBackend.CPU and self.cpu is not None:
            post = self.cpu.all_reduce_scaled(pre.cpu(), mass, 2 * self.round).to(pre.device)
            bpost = (self.cpu.all_reduce_scaled(bpre.cpu(), mover, 2 * self.round + 1).to(bpre.device)
                     if bpre is not None else None)
        else:
            tot = torch.tensor([mass, mover], dtype=torch.float64, device=pre.device)
            dist.all_reduce(tot)
            if float(tot[0]) <= 0.0:
                return 0.0  # nobody moved: the consensus already holds
            num = pre * (mass / float(tot[0]))
            dist.all_reduce(num)
            post = num
            bpost = None
            if bpre is not None:
                bnum = bpre * (mover / float(tot[1]))
                dist.all_reduce(bnum)
                bpost = bnum
        if self.alpha is not None:
            a = float(self.alpha)
            post = (1.0 - a) * pre + a * post
            if bpost is not None:
                bpost = (1.0 - a) * bpre + a * bpost
        _unflat_(self.params, post)
        if bpost is not None:
            self._load_buffers(bpost)
        return divergence(pre, post)

    def broadcast_initial(self) -> None:
        if self.world == 1:
            return
        if self.fused is not None:
            comm, arena = self.fused
            torch.cuda.synchronize(self.device)
            comm.broadcast_(arena.numel, root=0, slot=1)
            torch.cuda.synchronize(self.device)
            comm.check()
        else:
            for p in self.params:
                dist.broadcast(p.data, src=0)
        for b in self.model.buffers():
            if b.is_floating_point():
                dist.broadcast(b, src=0)

    def close(self) -> None:
        if self.fused is not None:
            self.fused[0].close()


def _rank_main(rank: int, world: int, port: int, key: bytes, spec: dict, out_q) -> None:
    """One training rank (a spawned process, or the caller for world == 1)."""
    try:
        dev_kind = spec["device_kind"]
        if world > 1:
            os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
            if dev_kind == "cuda":
                torch.cuda.set_device(rank)
                dist.init_process_group("nccl", rank=rank, world_size=world,
                                        timeout=datetime.timedelta(seconds=spec["timeout_s"]),
                                        device_id=torch.device("cuda", rank))
            else:
                dist.init_process_group("gloo", rank=rank, world_size=world,
                                        timeout=datetime.timedelta(seconds=spec["timeout_s"]))
        device = torch.device("cuda", rank) if dev_kind == "cuda" else torch.device("cpu")
        log.set_label(f"rank {rank}")
        state = _train_rank(rank, world, device, key, spec)
        if rank == 0:
            out_q.put(("ok", state))
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    except Exception as e:
        cfg = spec.get("config")
        if cfg is not None and getattr(cfg, "save_path_", None):
            try:  # forensic record next to the bundle, one file per rank
                from .bundle import CheckpointBundle, RankDeathRecord
                RankDeathRecord(rank, world, repr(e)).write_to_file(
                    CheckpointBundle.death_record_path(cfg.save_path_, rank))
            except OSError:
                pass
        out_q.put(("err", f"rank {rank}: " + traceback.format_exc()))


def _train_rank(rank, world, device, key, spec) -> TrainedState:
    cfg: TrainerConfig = spec["config"]
    ec: ElCheConfig = cfg.elche_
    policy, backend = ec.mode_.split()
    torch.manual_seed(spec.get("seed", 0))
    model = spec["model_factory"](device)
    opt = spec["optim_factory"](model.parameters())
    train_fn = spec["train_fn"]
    cpu_ctl = cpu_client = None
    if backend == AverageBackend.CPU and world > 1:
        from .cpu_reduce import CpuReduceClient, CpuReduceController

        port_t = torch.zeros(1, dtype=torch.int64, device=device if device.type == "cuda" else "cpu")
        if rank == 0:
            cpu_ctl = CpuReduceController(world, key, heartbeat_timeout=cfg.heartbeat_timeout_secs_)
            port_t[0] = cpu_ctl.port
        dist.broadcast(port_t, src=0)
        cpu_client = CpuReduceClient(rank, "127.0.0.1", int(port_t.item()), key)
    start_epoch, global_step = 0, 0
    if cfg.resume_from_:
        # every rank loads the same bundle; the initial broadcast then agrees anyway
        from .bundle import load_bundle
        meta = load_bundle(cfg.resume_from_, model, opt)
        start_epoch, global_step = meta.epoch + 1, meta.global_step
    # CpuAsync blends the consensus into each replica (EASGD); every other
    # mode overwrites with it (config.rs:283-313)
    alpha = ec.easgd_alpha_ if policy == ApplyPolicy.ASYNC else None
    avg = _Averager(model, opt, backend, rank, world, device, cpu_client, ec.gamma_, alpha)
    avg.broadcast_initial()
    sampler = DistributedSampler(rank, world, seed=spec.get("seed", 0))
    loader = (DataLoader.from_dataset(spec["dataset"]).batch_size(cfg.batch_size_).device(device)
              .sampler(sampler).build())
    native = None
    if policy == ApplyPolicy.CADENCE and world > 1:
        from .._ext import native as _native

        native = _native().ElChe(world, ec.anchor_)
        native.set_overhead_target(ec.overhead_target_)
        if ec.max_anchor_:
            native.set_max_anchor(ec.max_anchor_)
        native.set_min_anchor(ec.min_anchor_)
        if ec.max_batch_diff_:
            native.set_max_batch_diff(ec.max_batch_diff_)
        native.set_max_total(max(1, loader.num_batches() * world))
    guard = (NoGuard() if not ec.divergence_guard_ else LevelGuard(ec.divergence_threshold_))
    from .meta import LrEventMeta
    meta = LrEventMeta()
    outer = OuterStepper(spec.get("outer") or OuterAvg())
    st = TrainedState(world=world, mode=ec.mode_.value)
    counts = [1] * world if policy != ApplyPolicy.CADENCE else [ec.anchor_] * world
    st.start_epoch = start_epoch
    for epoch in range(start_epoch, cfg.num_epochs_):
        model.train()
        losses = []
        it = iter(loader.epoch(epoch))
        exhausted = False
        while not exhausted:
            window = counts[rank] if world > 1 else 1
            t0 = time.perf_counter()
            done = 0
            for _ in range(window):
                try:
                    batch = next(it)
                except StopIteration:
                    exhausted = True
                    break
                loss = train_fn(model, batch)
                loss.backward()
                if cfg.max_grad_norm_:
                    from ..nn.clip import clip_grad_norm

                    clip_grad_norm(model.parameters(), cfg.max_grad_norm_, opt)
                if cfg.scheduler_fn_ is not None:
                    opt.set_lr(cfg.scheduler_fn_(st.syncs))
                opt.step()
                opt.zero_grad()
                losses.append(float(loss.detach().float().item()))
                done += 1
                global_step += 1
            if device.type == "cuda":
                torch.cuda.synchronize(device)
            wall_ms = (time.perf_counter() - t0) * 1e3
            if world == 1:
                continue
            # every rank must enter the same number of averaging rounds; one
            # exchange carries (more data?, work done) of every rank
            flags = torch.tensor([0 if exhausted else 1, done], dtype=torch.int64,
                                 device=device if device.type == "cuda" else "cpu")
            allf = [torch.zeros_like(flags) for _ in range(world)]
            dist.all_gather(allf, flags)
            more = torch.tensor(min(int(f[0]) for f in allf))
            if sum(int(f[1]) for f in allf) == 0:
                # the cohort did no work in this window: skip the reduce
                break
            s0 = time.perf_counter()
            div = avg.average(done)
            sync_ms = (time.perf_counter() - s0) * 1e3
            st.syncs += 1
            st.divergence.append(div)
            if outer is not None and not isinstance(outer.opt, OuterAvg):
                flat = avg.flat()
                newg = outer.step(flat)
                if avg.fused is not None:
                    avg.fused[1].data.copy_(newg)
                    avg.fused[1].refresh_shadow()
                else:
                    _unflat_(avg.params, newg)
                if outer.opt.resets_inner:
                    opt.reset_state()
            if native is not None:
                t = torch.tensor([wall_ms, float(done)], dtype=torch.float64,
                                 device=device if device.type == "cuda" else "cpu")
                gathered = [torch.zeros_like(t) for _ in range(world)]
                dist.all_gather(gathered, t)
                verdict = guard.observe(div)
                if ec.meta_controller_:
                    lr_now = opt.lr() if hasattr(opt, "lr") else 0.0
                    f = meta.observe(lr_now, int(native.anchor()),
                                     "shrink" if verdict == Verdict.SHRINK else "ok", native.phase())
                    if f is not None:
                        native.nudge_anchor_down(f)
                        st.meta_nudges.append(f)
                native.report_timing([float(g[0]) for g in gathered],
                                     [int(g[1]) for g in gathered], sync_ms)
                counts = list(native.batch_counts())
                st.batch_counts.append(counts)
            if int(more.item()) == 0:
                exhausted = True
        if losses:
            st.losses.append(sum(losses) / len(losses))
        if cfg.epoch_fn_ is not None and rank == 0:
            cfg.epoch_fn_(epoch, model, st)
        if cfg.save_path_ and cfg.checkpoint_every_ and (epoch + 1) % cfg.checkpoint_every_ == 0 and rank == 0:
            from .bundle import save_bundle

            from .bundle import CheckpointMeta, ElCheState, SaveReason
            es = None
            if native is not None:
                ph = native.phase()
                es = ElCheState(int(native.anchor()), int(native.anchor_rank()),
                                [float(x) for x in native.ms_per_batch()],
                                ph.lower() if isinstance(ph, str) else
                                ("probe", "warmup", "stable", "mature")[int(ph)],
                                int(native.calibrations()))
            save_bundle(cfg.save_path_, model, opt,
                        CheckpointMeta(epoch, global_step, st.syncs, world, SaveReason.Checkpoint, es))
    st.params = [(n, p.detach().cpu().clone()) for n, p in model.named_parameters()]
    st.buffers = [(n, b.detach().cpu().clone()) for n, b in model.named_buffers()]
    avg.close()
    if cpu_client is not None:
        cpu_client.close()
    if cpu_ctl is not None:
        cpu_ctl.close()
    return st


class DdpHandle:
    def __init__(self, procs, q, inline_state=None):
        self.procs, self.q, self.inline_state = procs, q, inline_state

    def join(self, timeout: float = 3600.0) -> TrainedState:
        if self.inline_state is not None:
            return self.inline_state
        status, payload = self.q.get(timeout=timeout)
        for p in self.procs:
            p.join(timeout=120)
        if status != "ok":
            for p in self.procs:
                if p.is_alive():
                    p.terminate()
            raise RuntimeError(payload)
        return payload


class DdpBuilder:
    def __init__(self, model_factory, optim_factory, train_fn):
        self.spec: Dict[str, Any] = {"model_factory": model_factory, "optim_factory": optim_factory,
                                     "train_fn": train_fn, "config": TrainerConfig(),
                                     "timeout_s": 300.0, "seed": 0}
        self._devices: Optional[List[str]] = None

    def dataset(self, ds):
        self.spec["dataset"] = ds
        return self

    def config(self, cfg: TrainerConfig):
        self.spec["config"] = cfg
        return self

    def mode(self, m: ElCheMode):
        self.spec["config"].elche_.mode_ = m
        return self

    def outer(self, outer_opt):
        self.spec["outer"] = outer_opt
        return self

    def seed(self, s: int):
        self.spec["seed"] = s
        return self

    def devices(self, devs: List[str]):
        """e.g. ["cuda:0", "cuda:1"] or ["cpu"] * 2 (gloo ranks, for tests)."""
        self._devices = list(devs)
        return self

    def _resolve(self):
        if self._devices is not None:
            kinds = {torch.device(d).type for d in self._devices}
            if len(kinds) != 1:
                raise ValueError("all ranks must use one device kind")
            return len(self._devices), kinds.pop()
        n = torch.cuda.device_count()
        if n >= 2:
            return n, "cuda"  # auto-promote: one process per GPU
        return 1, "cuda" if n == 1 else "cpu"

    def run(self) -> DdpHandle:
        world, kind = self._resolve()
        self.spec["device_kind"] = kind
        key = os.urandom(16)
        if world == 1:
            q: "queue.Queue" = queue.Queue()
            _rank_main(0, 1, 0, key, self.spec, q)
            status, payload = q.get()
            if status != "ok":
                raise RuntimeError(payload)
            return DdpHandle([], None, payload)
        import torch.multiprocessing as mp

        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, key, self.spec, q), daemon=False)
                 for r in range(world)]
        for p in procs:
            p.start()
        return DdpHandle(procs, q)

    def into_worker(self, rank: Optional[int] = None, world: Optional[int] = None) -> "Worker":
        return Worker(self.spec, rank, world)


class Trainer:
    @staticmethod
    def builder(model_factory, optim_factory, train_fn) -> DdpBuilder:
        return DdpBuilder(model_factory, optim_factory, train_fn)

    @staticmethod
    def run(model_factory, optim_factory, train_fn, dataset, config: TrainerConfig) -> TrainedState:
        return (DdpBuilder(model_factory, optim_factory, train_fn).dataset(dataset).config(config)
                .run().join())


class Worker:
    """Cooperative tier (ddp_run/cooperative.rs): the user owns the loop.

        w = Trainer.builder(mf, of, tf).dataset(ds).into_worker()
        while (plan := w.next_plan()) is not None:
            for batch in plan:
                loss = my_step(w.model, batch); w.step(loss)
            w.sync()
        state = w.finish()

    Runs in the current process; rank/world come from torchrun's environment
    when not given.
    """

    def __init__(self, spec, rank=None, world=None):
        from .ddp import init_from_env

        r, wsz, local = init_from_env()
        self.rank = r if rank is None else rank
        self.world = wsz if world is None else world
        self.spec = spec
        cfg: TrainerConfig = spec["config"]
        self.device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
        self.model = spec["model_factory"](self.device)
        self.opt = spec["optim_factory"](self.model.parameters())
        self.avg = _Averager(self.model, self.opt, cfg.elche_.mode_.split()[1], self.rank,
                             self.world, self.device, None, cfg.elche_.gamma_)
        self.avg.broadcast_initial()
        self.loader = (DataLoader.from_dataset(spec["dataset"]).batch_size(cfg.batch_size_)
                       .device(self.device).sampler(DistributedSampler(self.rank, self.world)).build())
        self.epoch = 0
        self._it = None
        self.window = cfg.elche_.anchor_ if cfg.elche_.mode_.split()[0] == ApplyPolicy.CADENCE else 1
        self.done_in_window = 0
        self.state = TrainedState(world=self.world, mode=cfg.elche_.mode_.value)

    def next_plan(self):
        if self.epoch >= self.spec["config"].num_epochs_:
            return None
        if self._it is None:
            self._it = iter(self.loader.epoch(self.epoch))
        batches = []
        for _ in range(self.window):
            try:
                batches.append(next(self._it))
            except StopIteration:
                self._it = None
                self.epoch += 1
                break
        return batches

    def step(self, loss: torch.Tensor) -> None:
        loss.backward()
        self.opt.step()
        self.opt.zero_grad()
        self.done_in_window += 1
        self.state.losses.append(float(loss.detach().item()))

    def sync(self) -> float:
        div = self.avg.average(self.done_in_window)
        self.state.syncs += 1
        self.done_in_window = 0
        return div

    def finish(self) -> TrainedState:
        self.state.params = [(n, p.detach().cpu().clone()) for n, p in self.model.named_parameters()]
        self.avg.close()
        return self.state
