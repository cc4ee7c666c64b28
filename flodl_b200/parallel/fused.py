"""DDP with the fused peer-memory gradient all-reduce + optimizer update.

``FusedDdp(model, optimizer)`` re-homes the model's parameters, gradients and
bf16 weight shadows into symmetric peer-mapped arenas, broadcasts rank 0's
weights with the pull kernel, and cuts the arena into buckets. During
backward, the fused ops report each parameter's gradient as complete; when a
bucket is complete its fused kernel is launched on the communication stream
(overlapping the rest of backward): reduce-scatter over NVLink, AdamW/SGD on
this rank's shard, all-gather of the updated f32 weights and bf16 shadows into
every rank, gradient clear. Buckets below ``oneshot_kb`` run the one-shot form
instead (every rank reduces the whole bucket and updates it locally: no
all-gather, fewer bytes in flight, the lowest latency). ``finish()`` launches
what is left and joins the communication stream; there is no separate
``optimizer.step()`` or ``zero_grad()`` in this mode.

With ``max_grad_norm`` the buckets only reduce-scatter their gradients (the
average lands in this rank's shard, its sum of squares in an accumulator) and
``finish()`` launches one apply kernel that exchanges the partial sums, takes
the global norm, scales by ``max_norm / (norm + 1e-6)`` when the norm is above
``max_norm`` (the reference's ``clip_grad_norm``, flodl-sys/ops_training.cpp:
948-985) and then updates and all-gathers every bucket.

Several parameter groups (their own lr, weight decay, betas) share one
symmetric region: group k's arena is a slice of it, buckets never span two
groups, each bucket launch carries its group's hyper-parameters, and the
optimizer moments live in region-sized buffers (each group's state a view at
its base) because the kernels index state by region position. Global-norm
clipping is fused for a single group.

Semantics equal the reference's ``Ddp::wrap`` + ``all_reduce_gradients`` (Avg)
+ ``optimizer.step()`` (flodl/src/distributed/ddp.rs:249-260): every rank ends
the step with identical parameters. Optimizer moments of a two-shot bucket are
held only for the shard each rank owns (the other ranks' slices stay unused).
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..ops._common import add_grad_ready_listener, clear_grad_ready_listeners
from ..optim.optimizer import SGD, Adam, AdamW
from ..utils.arena import ParamArena
from .peer import PeerComm


class FusedDdp:
    fuses_optimizer = True

    def __init__(self, model: torch.nn.Module, optimizer, bucket_mb: Optional[float] = None,
                 blocks: int = 0, group=None, timeout_s: float = 10.0,
                 overlap_threads: Optional[int] = None, overlap_blocks: Optional[int] = None,
                 oneshot_kb: Optional[float] = None, tail_mb: Optional[float] = None,
                 max_grad_norm: Optional[float] = None):
        # tuning knobs (constructor arguments win over the environment):
        #   FLODL_DDP_BUCKET_MB        bucket size in MiB of f32 gradients (64)
        #   FLODL_DDP_TAIL_MB          size of the bucket holding the first parameters,
        #                              which completes last in backward (2)
        #   FLODL_DDP_ONESHOT_KB       buckets up to this size run the one-shot form (1024)
        #   FLODL_DDP_OVERLAP_THREADS  threads per CTA of in-backward launches (256)
        #   FLODL_DDP_OVERLAP_BLOCKS   CTAs of in-backward launches (0: two per SM)
        env = os.environ
        if bucket_mb is None:
            bucket_mb = float(env.get("FLODL_DDP_BUCKET_MB", "64"))
        if tail_mb is None:
            tail_mb = float(env.get("FLODL_DDP_TAIL_MB", "2"))
        if oneshot_kb is None:
            oneshot_kb = float(env.get("FLODL_DDP_ONESHOT_KB", "1024"))
        if overlap_threads is None:
            overlap_threads = int(env.get("FLODL_DDP_OVERLAP_THREADS", "256"))
        if overlap_blocks is None:
            overlap_blocks = int(env.get("FLODL_DDP_OVERLAP_BLOCKS", "0"))
        self.model = model
        self.opt = optimizer
        self.groups = list(optimizer.groups)
        self.group = self.groups[0]
        params = [p for g in self.groups for p in g.params]
        self.params = params
        self.device = params[0].device
        self.max_grad_norm = float(max_grad_norm) if max_grad_norm else 0.0
        if self.max_grad_norm and len(self.groups) > 1:
            raise ValueError("FusedDdp: global-norm clipping is fused for one parameter group; "
                             "use one group or clip outside the fused path")
        sizes = [sum((p.numel() + 63) // 64 * 64 for p in g.params) for g in self.groups]
        numel = sum(sizes)
        self.comm = PeerComm(numel, self.device, group=group, timeout_s=timeout_s)
        self.rank, self.world = self.comm.rank, self.comm.world
        # one symmetric region for every group: group k's arena is the slice
        # [base_k, base_k + size_k) of the peer-mapped data/grad/shadow regions
        self.arenas: List[ParamArena] = []
        self.bases: List[int] = []
        base = 0
        for g, n in zip(self.groups, sizes):
            lo = base
            arena = ParamArena(g.params,
                               alloc=lambda k, dt, dv, lo=lo: self.comm.data[lo:lo + k],
                               grad_alloc=lambda k, dt, dv, lo=lo: self.comm.grad[lo:lo + k],
                               with_shadow=False)
            arena.shadow = self.comm.shadow[lo:lo + arena.numel]
            arena.rebind()
            arena.refresh_shadow()
            g.arena = arena
            self.arenas.append(arena)
            self.bases.append(lo)
            base += n
        self.arena = self.arenas[0]
        self.numel = base
        self.blocks = blocks
        self.overlap_threads = overlap_threads
        self.overlap_blocks = overlap_blocks or 2 * self.comm.C.num_sms()
        self.oneshot_elems = int(oneshot_kb * 1024 / 4)
        self.kind = "adamw" if isinstance(optimizer, Adam) else "sgd" if isinstance(optimizer, SGD) else None
        if self.kind is None:
            raise ValueError("FusedDdp supports Adam/AdamW and SGD")
        # optimizer state (device scalars per group; moments over the whole
        # region, each group's state a view at its base, because the kernels
        # index state by the element's position in the region)
        for g in self.groups:
            optimizer._device_scalars(g)
            if (isinstance(optimizer, Adam) and not isinstance(optimizer, AdamW)
                    and g.hyper["weight_decay"]):
                raise ValueError("FusedDdp: Adam with L2 weight decay is not fused; use AdamW")
            optimizer._init_fused_state(g)
        self._state = {}
        names = ("m", "v") if self.kind == "adamw" else ("buf",)
        for name in names:
            if any(getattr(g, name, None) is None for g in self.groups):
                continue  # SGD without momentum keeps no buffer
            whole = torch.zeros(self.numel, device=self.device, dtype=torch.float32)
            for g, lo in zip(self.groups, self.bases):
                part = whole[lo:lo + g.arena.numel]
                part.copy_(getattr(g, name))
                setattr(g, name, part)
            self._state[name] = whole
        if self.kind == "adamw":
            # step_t holds the number of the update the next bucket kernels apply
            for g in self.groups:
                self.comm.C.add_scalar(g.step_t, 1.0)
        self.comm_stream = torch.cuda.Stream(self.device)
        self._build_buckets(bucket_mb, tail_mb)
        if self.max_grad_norm:
            self.sumsq = torch.zeros(1, dtype=torch.float32, device=self.device)
            self.grad_norm = torch.zeros(1, dtype=torch.float32, device=self.device)
            self.table = torch.tensor([[b["start"], b["end"]] for b in self.buckets],
                                      dtype=torch.int64, device=self.device)
        for p in params:
            clear_grad_ready_listeners(p)
            add_grad_ready_listener(p, self._on_ready)
        # initial state: rank 0's parameters on every rank (pull broadcast)
        torch.cuda.synchronize(self.device)
        self.comm.broadcast_(self.numel, root=0, slot=self._slot_bcast, blocks=blocks)
        torch.cuda.synchronize(self.device)
        self.comm.check()
        if self.world > 1:
            for b in model.buffers():
                if b.is_floating_point():
                    dist.broadcast(b, src=0)
        self._launched: set = set()

    def _build_buckets(self, bucket_mb: float, tail_mb: float) -> None:
        """Buckets over the region in forward parameter order, never spanning
        two parameter groups: the first (holding the earliest parameters,
        whose gradients complete last) is capped at ``tail_mb``, the others at
        ``bucket_mb``; they launch in reverse order as backward completes
        them."""
        caps = (int(tail_mb * (1 << 20) / 4), int(bucket_mb * (1 << 20) / 4))
        chunks: List[tuple] = []  # (group index, [param indices])
        for gi, a in enumerate(self.arenas):
            cur, size = [], 0
            for i in range(len(a.params)):
                n = a.params[i].numel()
                cap = caps[0] if not chunks else caps[1]
                if cur and size + n > cap:
                    chunks.append((gi, cur))
                    cur, size = [], 0
                cur.append(i)
                size += n
            if cur:
                chunks.append((gi, cur))
        self.buckets: List[dict] = []
        self._bucket_of: Dict[int, dict] = {}
        for gi, idx in reversed(chunks):
            self._close(gi, idx)
        self._slot_bcast = len(self.buckets)
        self._slot_avg = self._slot_bcast + 1
        self._slot_apply = self._slot_bcast + 2
        if self._slot_apply >= self.comm.C.MAX_SLOTS:
            raise ValueError("too many buckets; raise bucket_mb")

    def _close(self, gi: int, idx: List[int]) -> None:
        a, base = self.arenas[gi], self.bases[gi]
        start = base + min(a.offsets[i] for i in idx)
        end = base + max(a.offsets[i] + ((a.params[i].numel() + 63) // 64) * 64 for i in idx)
        b = {"slot": len(self.buckets), "start": start, "end": end, "group": gi,
             "params": [a.params[i] for i in idx], "pending": len(idx),
             "oneshot": (end - start) <= self.oneshot_elems and not self.max_grad_norm}
        self.buckets.append(b)
        for i in idx:
            self._bucket_of[id(a.params[i])] = b

    def _on_ready(self, p) -> None:
        b = self._bucket_of.get(id(p))
        if b is None:
            return
        b["pending"] -= 1
        if b["pending"] == 0:
            self._launch(b)

    def _update_args(self, gi: int = 0) -> dict:
        """Hyper-parameters of group gi; the state buffers are those of the
        whole region (the kernels index them by region position)."""
        g = self.groups[gi]
        h = g.hyper
        if self.kind == "adamw":
            return dict(m=self._state["m"], v=self._state["v"], lr=g.lr_t, step=g.step_t,
                        gscale=self.opt.gscale_t, beta1=h["beta1"], beta2=h["beta2"],
                        eps=h["eps"], wd=h["weight_decay"])
        return dict(m=self._state.get("buf"), lr=g.lr_t, first=g.first_t,
                    gscale=self.opt.gscale_t, wd=h["weight_decay"], momentum=h["momentum"],
                    dampening=h["dampening"], nesterov=int(h["nesterov"]))

    def _launch(self, b, tail: bool = False) -> None:
        """Launch bucket b's fused kernel on the communication stream. Buckets
        that complete during backward run a grid of small CTAs that fits beside
        the compute kernels' CTAs, so the collective overlaps backward; the
        tail launched by finish() takes the full grid."""
        cur = torch.cuda.current_stream(self.device)
        self.comm_stream.wait_stream(cur)
        if tail:
            geo = {"blocks": self.blocks, "threads": 512}
        else:
            geo = {"blocks": self.overlap_blocks, "threads": self.overlap_threads}
        C = self.comm.C
        with torch.cuda.stream(self.comm_stream):
            if self.max_grad_norm:
                self.comm.launch(C.FUSED_REDUCE_SCATTER, bucket=b["slot"], start=b["start"],
                                 end=b["end"], sumsq=self.sumsq, gscale=self.opt.gscale_t, **geo)
            else:
                op = C.FUSED_AR_ADAMW if self.kind == "adamw" else C.FUSED_AR_SGD
                self.comm.launch(op, bucket=b["slot"], start=b["start"], end=b["end"],
                                 oneshot=int(b["oneshot"]), **self._update_args(b["group"]),
                                 **geo)
        self._launched.add(b["slot"])

    def finish(self) -> None:
        """Launch buckets not yet reported ready, then join the comm stream."""
        for b in self.buckets:
            if b["slot"] not in self._launched:
                self._launch(b, tail=True)
        if self.max_grad_norm:
            C = self.comm.C
            op = C.FUSED_CLIP_APPLY_ADAMW if self.kind == "adamw" else C.FUSED_CLIP_APPLY_SGD
            args = self._update_args()
            args.pop("gscale", None)  # the buckets already applied it
            with torch.cuda.stream(self.comm_stream):
                self.comm.launch(op, bucket=self._slot_apply, start=0, end=0, sumsq=self.sumsq,
                                 norm_out=self.grad_norm, max_norm=self.max_grad_norm,
                                 table=self.table, nb=len(self.buckets), blocks=self.blocks,
                                 threads=512, **args)
        torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)
        for g in self.groups:
            if self.kind == "adamw":
                self.comm.C.add_scalar(g.step_t, 1.0)
            else:
                g.first_t.zero_()
        for b in self.buckets:
            b["pending"] = len(b["params"])
        self._launched = set()

    all_reduce_gradients = finish

    def average_params(self, mass: float = 1.0) -> None:
        """Weighted parameter average across ranks (cluster averaging);
        ``mass`` is this rank's gamma-mass."""
        self.comm.weighted_average_(self.numel, mass, slot=self._slot_avg,
                                    blocks=self.blocks)

    def close(self) -> None:
        self.comm.close()
