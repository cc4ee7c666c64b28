"""Managed (``Trainer``) and cooperative (``into_worker``) training tiers.

Reference: ``Trainer::builder(model_factory, optim_factory, train_fn)`` ->
``DdpBuilder`` -> ``.run()`` -> ``DdpHandle::join()`` -> ``TrainedState``
(flodl/src/distributed/ddp.rs:408-560, ddp_run/*). With two or more devices
(or ``devices([...])``) the trainer runs one process per rank under a cluster
coordinator (``parallel/runtime.py``) hosted by the launching process: the
coordinator dispatches each rank's window from the epoch's chunk pool, decides
when the ranks average, feeds the timings to ElChe and the divergence to the
convergence guard, and re-forms the survivors when a rank leaves or stops
answering. Averaging follows the ``ElCheMode``:

* Sync:    every rank steps its optimizer, then parameters (work-weighted)
           and f32 buffers (mean over the ranks that moved) are averaged
           every window of one step.
* Cadence: rank r runs ``batch_counts[r]`` steps per window (ElChe balances
           the counts from measured ms/batch and the averaging overhead), then
           the work-weighted average ``sum_r n_r^gamma W_r / sum n^gamma``.
* Async (CPU backend): ranks that finish early keep training for up to
           ``max_overshoot`` batches, and each rank blends the consensus into
           its replica (EASGD, ``easgd_alpha``) instead of overwriting.

Device averaging runs the fused peer-memory weighted-average kernel on CUDA
(the mass exchange rides its signal words, the divergence partials come back
with it); on CPU ranks it is a gloo all-reduce. The CPU backend goes through
the signed-frame CPU reducer that the coordinator hosts. Each session's
process group is gloo (bootstrap only: the device data path is the peer
kernels), so survivors can re-form without a device communicator abort. A
round that fails (a peer wait ran out, a collective timed out) is retried on
the re-formed session after every rank restored its pre-round parameters.
Outer optimizers (SlowMo / DiLoCo) apply to each consensus.

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
    record: Dict[str, Any] = field(default_factory=dict)  # the coordinator's run record


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
            self._make_fused()

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

    def snapshot(self) -> None:
        """Keep this rank's pre-round parameters and buffers (restored when a
        round fails, before it is retried on a re-formed session)."""
        with torch.no_grad():
            self._pre = self.flat()
            self._pre_buf = self._buffers_flat()

    def restore(self) -> None:
        pre = getattr(self, "_pre", None)
        if pre is None:
            return
        with torch.no_grad():
            if self.fused is not None:
                self.fused[1].data.copy_(pre)
                self.fused[1].refresh_shadow()
            else:
                _unflat_(self.params, pre)
            if self._pre_buf is not None:
                self._load_buffers(self._pre_buf)

    def rebuild(self, rank: int, world: int) -> None:
        """Re-form over the current default process group (a survivor set):
        a new symmetric region holds the parameters, the old communicator is
        abandoned without touching any peer's memory."""
        self.rank, self.world = rank, world
        if self.fused is None:
            return
        old_comm, old_arena = self.fused
        torch.cuda.synchronize(self.device)
        self.fused = None
        if world > 1:
            self._make_fused()
        else:
            # alone: the parameters move to private memory
            from ..utils.arena import ParamArena
            arena = ParamArena(self.params)
            for g in self.opt.groups:
                if getattr(g, "arena", None) is old_arena:
                    self.opt.adopt_arena(g, arena)
        old_comm.abandon()

    def _make_fused(self) -> None:
        from ..utils.arena import ParamArena
        from .peer import PeerComm

        nparam = sum((p.numel() + 63) // 64 * 64 for p in self.params)
        self.nbuf = sum(b.numel() for b in self.buffers)
        comm = PeerComm(nparam + (self.nbuf + 63) // 64 * 64, self.device)
        arena = ParamArena(self.params, alloc=comm.data_alloc, grad_alloc=comm.grad_alloc,
                           with_shadow=False)
        arena.shadow = comm.shadow[:arena.numel]
        arena.rebind()
        arena.refresh_shadow()
        self.fused = (comm, arena)
        self.buf_start = arena.numel
        self.buf_view = comm.data[self.buf_start:self.buf_start + self.nbuf]
        self.div = torch.zeros(2, dtype=torch.float32, device=self.device)
        opt = self.opt
        for g in opt.groups:
            if all(any(q is p for q in arena.params) for p in g.params) and len(opt.groups) == 1:
                opt.adopt_arena(g, arena)

    def average(self, batches: int, rnd: Optional[int] = None) -> float:
        """Average with this rank's work; returns ||pre - post|| / ||post||.
        ``rnd`` names the round for the CPU reducer (every rank passes the same)."""
        mass = realized_mass(batches, self.gamma)
        mover = 1.0 if batches > 0 else 0.0
        self.round += 1
        rnd = self.round if rnd is None else int(rnd)
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
            post = self.cpu.all_reduce_scaled(pre.cpu(), mass, 2 * rnd).to(pre.device)
            bpost = (self.cpu.all_reduce_scaled(bpre.cpu(), mover, 2 * rnd + 1).to(bpre.device)
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


class _Bytes:
    """A tensor pickled by value (dtype, shape, raw bytes)."""

    def __init__(self, t: torch.Tensor):
        t = t.detach().cpu().contiguous()
        self.dtype = str(t.dtype).split(".")[-1]
        self.shape = tuple(t.shape)
        self.data = t.reshape(-1).view(torch.uint8).numpy().tobytes()

    def tensor(self) -> torch.Tensor:
        raw = torch.frombuffer(bytearray(self.data), dtype=torch.uint8)
        return raw.view(getattr(torch, self.dtype)).reshape(self.shape)


def _report_by_value(st: "TrainedState") -> "TrainedState":
    """Tensors of a rank's report pickled by value: a queue would otherwise
    pass them as shared-memory handles that die with the rank process, which
    may exit before the parent reads them."""
    st.params = [(n, _Bytes(t) if isinstance(t, torch.Tensor) else t) for n, t in st.params]
    st.buffers = [(n, _Bytes(t) if isinstance(t, torch.Tensor) else t) for n, t in st.buffers]
    return st


def _report_as_tensors(st: "TrainedState") -> "TrainedState":
    st.params = [(n, t.tensor() if isinstance(t, _Bytes) else t) for n, t in st.params]
    st.buffers = [(n, t.tensor() if isinstance(t, _Bytes) else t) for n, t in st.buffers]
    return st


def _rank_main(rank: int, world: int, host: str, port: int, key: bytes, spec: dict,
               out_q) -> None:
    """One training rank process: follows the coordinator's control messages."""
    try:
        device = (torch.device("cuda", rank) if spec["device_kind"] == "cuda"
                  else torch.device("cpu"))
        if device.type == "cuda":
            torch.cuda.set_device(device)
        log.set_label(f"rank {rank}")
        report = _RankWorker(rank, world, host, port, key, spec, device).run()
        if report is not None:
            out_q.put(("ok", _report_by_value(report)))
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
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


class _RankWorker:
    """The GpuWorker role (ddp_run/worker/*): model and optimizer replica, the
    training of dispatched windows, averaging rounds with restore-and-retry,
    session re-formation and epoch callbacks."""

    def __init__(self, rank, world, host, port, key, spec, device):
        from .runtime import RankAgent

        self.rank, self.world, self.spec, self.device = rank, world, spec, device
        self.key = key
        cfg: TrainerConfig = spec["config"]
        self.cfg = cfg
        ec = cfg.elche_
        self.policy, self.backend = ec.mode_.split()
        torch.manual_seed(spec.get("seed", 0))
        self.model = spec["model_factory"](device)
        self.opt = spec["optim_factory"](self.model.parameters())
        self.train_fn = spec["train_fn"]
        self.global_step = 0
        if cfg.resume_from_:
            from .bundle import load_bundle
            meta = load_bundle(cfg.resume_from_, self.model, self.opt)
            self.global_step = meta.global_step
        self.loader = (DataLoader.from_dataset(spec["dataset"]).batch_size(cfg.batch_size_)
                       .device(device).build())
        self.seed = spec.get("seed", 0)
        self.avg: Optional[_Averager] = None
        self.cpu_client = None
        self.since_sync = 0
        self.windows = 0
        self.syncs = 0
        self.epoch_losses: List[float] = []
        self._loss_sum = 0.0
        self._loss_n = 0
        self.divs: List[float] = []
        self.outer = OuterStepper(spec.get("outer") or OuterAvg())
        hb = max(0.05, min(1.0, cfg.heartbeat_timeout_secs_ / 5.0))
        self.agent = RankAgent(host, port, key, rank, heartbeat_s=hb)
        hooks = spec.get("test_hooks") or {}
        self.leave_after = (hooks.get("leave_after_syncs") or {}).get(rank)
        self.hang_after = (hooks.get("hang_after_windows") or {}).get(rank)
        self.slow_ms = (hooks.get("slow_ms_per_batch") or {}).get(rank, 0.0)

    # -------------------------------------------------------------- control loop
    def run(self) -> Optional[TrainedState]:
        from .runtime import (K_DEAD, K_DONE, K_EPOCH, K_EPOCH_ACK, K_PLAN, K_REBUILT,
                              K_SESSION, K_STOP, K_SYNC, K_SYNCED)
        try:
            while True:
                kind, body = self.agent.recv()
                if kind == K_SESSION:
                    self._session(body)
                    self.agent.send(K_REBUILT, {"session": body["session"]})
                elif kind == K_PLAN:
                    self.agent.send(K_DONE, self._train(body))
                    self.windows += 1
                    if self.hang_after is not None and self.windows >= self.hang_after:
                        self.agent.pause_heartbeat()  # a rank that stops answering
                        while True:
                            time.sleep(3600)
                elif kind == K_SYNC:
                    self.agent.send(K_SYNCED, self._sync(body))
                    if self.leave_after is not None and self.syncs >= self.leave_after:
                        # leave between windows: nothing of ours is in flight
                        if self.device.type == "cuda":
                            torch.cuda.synchronize(self.device)
                        self.agent.close(bye=True)
                        self._close()
                        return None
                elif kind == K_EPOCH:
                    self._epoch_end(body)
                    self.agent.send(K_EPOCH_ACK, {"epoch": body["epoch"]})
                elif kind == K_DEAD:
                    log.verbose(f"rank {body.get('rank')} declared dead")
                elif kind == K_STOP:
                    if body.get("error"):
                        raise RuntimeError(f"coordinator stopped the run: {body['error']}")
                    if body.get("report_rank") == self.rank:
                        return self._report()
                    return None
        finally:
            self._close()

    def _close(self) -> None:
        if self.avg is not None:
            try:
                if self.avg.fused is not None:
                    self.avg.fused[0].abandon()
                    self.avg.fused = None
            except Exception:
                pass
        if self.cpu_client is not None:
            try:
                self.cpu_client.close()
            except Exception:
                pass
            self.cpu_client = None
        try:
            self.agent.close()
        except Exception:
            pass

    # -------------------------------------------------------------- session
    def _session(self, body: dict) -> None:
        ranks = [int(r) for r in body["ranks"]]
        me, n = ranks.index(self.rank), len(ranks)
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass
        dist.init_process_group(
            "gloo", init_method=f"tcp://127.0.0.1:{int(body['port'])}", rank=me, world_size=n,
            timeout=datetime.timedelta(seconds=float(self.spec.get("group_timeout_s", 60.0))))
        if self.backend == AverageBackend.CPU and self.cpu_client is None and body.get("cpu_port"):
            from .cpu_reduce import CpuReduceClient
            self.cpu_client = CpuReduceClient(self.rank, "127.0.0.1", int(body["cpu_port"]), self.key)
        if self.avg is None:
            alpha = self.cfg.elche_.easgd_alpha_ if self.policy == ApplyPolicy.ASYNC else None
            self.avg = _Averager(self.model, self.opt, self.backend, me, n, self.device,
                                 self.cpu_client, self.cfg.elche_.gamma_, alpha)
            self.avg.broadcast_initial()
        else:
            self.avg.rebuild(me, n)
            self.avg.cpu = self.cpu_client

    # -------------------------------------------------------------- training
    def _train(self, plan: dict) -> dict:
        from ..data.sampler import ChunkSampler
        cfg = self.cfg
        self.loader.sampler_ = ChunkSampler([(a, a + n) for a, n in plan["spans"]], self.seed)
        limit = int(plan["batches"])
        self.model.train()
        dev = self.device
        t0 = time.perf_counter()
        first_ms = None
        n = samples = 0
        loss_acc = torch.zeros((), dtype=torch.float32, device=dev)
        for batch in self.loader.epoch(int(plan["epoch"])):
            if n >= limit:
                break
            loss = self.train_fn(self.model, batch)
            loss.backward()
            if cfg.max_grad_norm_:
                from ..nn.clip import clip_grad_norm
                clip_grad_norm(self.model.parameters(), cfg.max_grad_norm_, self.opt)
            if cfg.scheduler_fn_ is not None:
                self.opt.set_lr(cfg.scheduler_fn_(self.syncs))
            self.opt.step()
            self.opt.zero_grad()
            loss_acc += loss.detach().float()
            n += 1
            self.global_step += 1
            b0 = batch[0] if isinstance(batch, (list, tuple)) else next(iter(batch))
            samples += int(b0.shape[0])
            if self.slow_ms:
                time.sleep(self.slow_ms / 1e3)
            if first_ms is None:
                if dev.type == "cuda":
                    torch.cuda.synchronize(dev)
                first_ms = (time.perf_counter() - t0) * 1e3
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        wall = (time.perf_counter() - t0) * 1e3
        ls = float(loss_acc.item())
        self._loss_sum += ls
        self._loss_n += n
        self.since_sync += n
        return {"wid": plan["wid"], "batches": n, "samples": samples, "wall_ms": wall,
                "first_ms": first_ms or 0.0, "loss_sum": ls, "n_loss": n}

    # -------------------------------------------------------------- averaging
    def _sync(self, body: dict) -> dict:
        rnd = int(body["round"]) * 64 + int(body.get("attempt", 1))
        t0 = time.perf_counter()
        ok, err, div = True, None, 0.0
        self.avg.snapshot()
        try:
            div = self.avg.average(self.since_sync, rnd=rnd)
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
        except Exception as e:  # a peer timeout or a process-group error
            ok, err = False, repr(e)
            self.avg.restore()
        sync_ms = (time.perf_counter() - t0) * 1e3
        if ok:
            self.since_sync = 0
            self.syncs += 1
            self.divs.append(div)
            if not isinstance(self.outer.opt, OuterAvg):
                flat = self.avg.flat()
                newg = self.outer.step(flat)
                if self.avg.fused is not None:
                    self.avg.fused[1].data.copy_(newg)
                    self.avg.fused[1].refresh_shadow()
                else:
                    _unflat_(self.avg.params, newg)
                if self.outer.opt.resets_inner:
                    self.opt.reset_state()
        lr = self.opt.lr() if hasattr(self.opt, "lr") else 0.0
        return {"round": body["round"], "ok": ok, "err": err, "sync_ms": sync_ms, "div": div,
                "lr": float(lr)}

    # -------------------------------------------------------------- epochs
    def _epoch_end(self, body: dict) -> None:
        epoch = int(body["epoch"])
        if self._loss_n:
            self.epoch_losses.append(self._loss_sum / self._loss_n)
        self._loss_sum, self._loss_n = 0.0, 0
        mine = int(body.get("callback_rank", 0)) == self.rank
        if mine and self.cfg.epoch_fn_ is not None:
            self.cfg.epoch_fn_(epoch, self.model, self._report())
        if mine and body.get("save") and self.cfg.save_path_:
            from .bundle import (CheckpointMeta, CoverageBlock, ElCheState, EpochCoverage,
                                 SaveReason, save_bundle)
            es = body.get("elche_state")
            st = ElCheState(int(es["anchor"]), es["anchor_rank"],
                            [float(x) for x in es["smoothed_ms_per_batch"]], es["phase"],
                            int(es["calibration_count"])) if es else None
            cov = CoverageBlock(self.seed, self.cfg.batch_size_,
                                [EpochCoverage(epoch, len(self.spec["dataset"]),
                                               [tuple(r) for r in body.get("coverage", [])])])
            save_bundle(self.cfg.save_path_, self.model, self.opt,
                        CheckpointMeta(epoch, self.global_step, int(body.get("syncs", 0)),
                                       self.world, SaveReason.Checkpoint, st, cov))

    def _report(self) -> TrainedState:
        st = TrainedState(world=self.world, mode=self.cfg.elche_.mode_.value)
        st.params = [(n, p.detach().cpu().clone()) for n, p in self.model.named_parameters()]
        st.buffers = [(n, b.detach().cpu().clone()) for n, b in self.model.named_buffers()]
        st.losses = list(self.epoch_losses)
        st.syncs = self.syncs
        st.divergence = list(self.divs)
        return st


def _train_single(spec) -> TrainedState:
    """One device, no averaging: the single-device fallback of the trainer."""
    cfg: TrainerConfig = spec["config"]
    dev = (torch.device("cuda", 0) if spec["device_kind"] == "cuda" else torch.device("cpu"))
    torch.manual_seed(spec.get("seed", 0))
    model = spec["model_factory"](dev)
    opt = spec["optim_factory"](model.parameters())
    start_epoch, global_step = 0, 0
    if cfg.resume_from_:
        from .bundle import load_bundle
        meta = load_bundle(cfg.resume_from_, model, opt)
        start_epoch, global_step = meta.epoch + 1, meta.global_step
    loader = (DataLoader.from_dataset(spec["dataset"]).batch_size(cfg.batch_size_).device(dev)
              .seed(spec.get("seed", 0)).build())
    st = TrainedState(world=1, mode=cfg.elche_.mode_.value, start_epoch=start_epoch)
    for epoch in range(start_epoch, cfg.num_epochs_):
        model.train()
        acc = torch.zeros((), device=dev)
        n = 0
        for batch in loader.epoch(epoch):
            loss = spec["train_fn"](model, batch)
            loss.backward()
            if cfg.max_grad_norm_:
                from ..nn.clip import clip_grad_norm
                clip_grad_norm(model.parameters(), cfg.max_grad_norm_, opt)
            if cfg.scheduler_fn_ is not None:
                opt.set_lr(cfg.scheduler_fn_(global_step))
            opt.step()
            opt.zero_grad()
            acc += loss.detach().float()
            n += 1
            global_step += 1
        if n:
            st.losses.append(float(acc.item()) / n)
        if cfg.epoch_fn_ is not None:
            cfg.epoch_fn_(epoch, model, st)
        if cfg.save_path_ and cfg.checkpoint_every_ and (epoch + 1) % cfg.checkpoint_every_ == 0:
            from .bundle import CheckpointMeta, SaveReason, save_bundle
            save_bundle(cfg.save_path_, model, opt,
                        CheckpointMeta(epoch, global_step, 0, 1, SaveReason.Checkpoint, None))
    st.params = [(n_, p.detach().cpu().clone()) for n_, p in model.named_parameters()]
    st.buffers = [(n_, b.detach().cpu().clone()) for n_, b in model.named_buffers()]
    return st


class DdpHandle:
    """A running job: ``join()`` waits for it and returns the trained state
    with the coordinator's record (batch counts, divergence, verdicts, deaths)."""

    def __init__(self, procs, q, inline_state=None, coordinator=None):
        self.procs, self.q, self.inline_state = procs, q, inline_state
        self.coordinator = coordinator

    def join(self, timeout: float = 3600.0) -> TrainedState:
        if self.inline_state is not None:
            return self.inline_state
        import queue as _queue
        deadline = time.time() + timeout
        status = payload = None
        while status is None:
            try:
                status, payload = self.q.get(timeout=1.0)
            except _queue.Empty:
                if self.coordinator is not None and self.coordinator._done.is_set() \
                        and self.coordinator.error:
                    status, payload = "err", self.coordinator.error
                elif time.time() > deadline:
                    status, payload = "err", "training did not finish in time"
        rec = None
        if self.coordinator is not None:
            try:
                rec = self.coordinator.result(timeout=60)
            except RuntimeError as e:
                if status == "ok":
                    status, payload = "err", str(e)
        for p in self.procs:
            p.join(timeout=30)
        for p in self.procs:
            if p.is_alive():
                p.terminate()  # a rank the test told to hang
                p.join(timeout=10)
        if status != "ok":
            raise RuntimeError(payload)
        st: TrainedState = _report_as_tensors(payload)
        if rec is not None:
            st.world = self.coordinator.world
            st.syncs = rec["syncs"]
            st.batch_counts = rec["batch_counts"]
            st.divergence = rec["divergence"]
            st.meta_nudges = rec.get("meta_nudges", [])
            st.start_epoch = self.coordinator.start_epoch
            st.record = rec
        return st


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
            return DdpHandle([], None, _train_single(self.spec))
        import torch.multiprocessing as mp
        from .runtime import Coordinator

        ds = self.spec.get("dataset")
        if ds is None:
            raise ValueError("DdpBuilder: dataset(...) is required")
        coord = Coordinator(world, key, len(ds), self.spec["config"],
                            seed=self.spec.get("seed", 0)).start()
        host, port = coord.address()
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        procs = [ctx.Process(target=_rank_main, args=(r, world, host, port, key, self.spec, q),
                             daemon=False) for r in range(world)]
        for p in procs:
            p.start()
        return DdpHandle(procs, q, coordinator=coord)

    def test_hooks(self, **hooks):
        """Failure-injection seams for tests, all on the host: ``leave_after_syncs``
        {rank: n} (the rank leaves cleanly after its n-th averaging round),
        ``hang_after_windows`` {rank: n} (the rank stops heart-beating and
        sleeps), ``slow_ms_per_batch`` {rank: ms}."""
        self.spec["test_hooks"] = hooks
        return self

    def group_timeout(self, seconds: float):
        """Timeout of the per-session process group (a collective with a lost
        peer fails after it and the round is retried on the survivors)."""
        self.spec["group_timeout_s"] = float(seconds)
        return self

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
