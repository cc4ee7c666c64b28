"""Optimizers (flodl/src/nn/optim/*.rs).

Semantics follow floDl: ``step()``, ``zero_grad()``, ``lr()``/``set_lr()``,
``set_group_lr()``, ``scale_lr()``, ``reset_state()`` (used by DiLoCo),
parameter groups, and ``.optim`` state files (``FDLO | version | kind`` header,
then a per-optimizer payload, optional gzip, atomic write).

CUDA execution: each parameter group is re-homed into a flat arena
(:class:`~flodl_b200.utils.arena.ParamArena`) on the first step and updated by
ONE fused sm_100a kernel (AdamW / SGD-momentum) that also refreshes the bf16
weight shadow and can zero the gradient. lr and the step counter live in device
scalars, so a CUDA graph that captured ``step()`` replays correctly. The CPU
path applies the same math with ATen ops.
"""
from __future__ import annotations

import gzip
import io
import math
import os
import struct
from typing import Dict, Iterable, List, Optional, Sequence

import torch

from .._ext import cuda_ext, native
from ..utils.arena import ParamArena, arena_of

STATE_MAGIC = b"FDLO"
STATE_VERSION = 1
KIND_TAGS = {"SGD": 1, "Adam": 2, "AdamW": 3, "RMSprop": 4, "Adagrad": 5, "RAdam": 6,
             "NAdam": 7, "GradScaler": 8}
_DTYPE_FROM_TAG = {1: torch.float16, 2: torch.bfloat16, 3: torch.float32, 4: torch.float64,
                   5: torch.int32, 6: torch.int64}


# ------------------------------------------------------------------ state IO helpers
def write_tensor_state(w: io.BufferedIOBase, t: Optional[torch.Tensor]) -> None:
    w.write(native().encode_tensor_state(t))


def read_tensor_state(r, device) -> Optional[torch.Tensor]:
    present = r.read(1)
    if not present or present[0] == 0:
        return None
    (nd,) = struct.unpack("<I", r.read(4))
    shape = struct.unpack(f"<{nd}q", r.read(8 * nd)) if nd else ()
    tag = r.read(1)[0]
    (nbytes,) = struct.unpack("<Q", r.read(8))
    raw = bytearray(r.read(nbytes))
    dt = _DTYPE_FROM_TAG[tag]
    t = torch.frombuffer(raw, dtype=dt).reshape(shape) if nbytes else torch.empty(shape, dtype=dt)
    return t.clone().to(device)


def _atomic_write(path: str, payload: bytes) -> None:
    tmp = path + ".tmp"
    try:
        if path.endswith(".gz"):
            with gzip.open(tmp, "wb") as f:
                f.write(payload)
        else:
            with open(tmp, "wb") as f:
                f.write(payload)
        os.replace(tmp, path)
    except BaseException:
        if os.path.exists(tmp):
            os.remove(tmp)
        raise


def _open_read(path: str):
    return gzip.open(path, "rb") if path.endswith(".gz") else open(path, "rb")


class ParamGroup:
    def __init__(self, params: List[torch.Tensor], lr: float, **hyper):
        self.params = params
        self.lr = float(lr)
        self.hyper = hyper
        self.arena: Optional[ParamArena] = None
        self.lr_t: Optional[torch.Tensor] = None
        self.lr_t_val: Optional[float] = None
        self.step_t: Optional[torch.Tensor] = None


class Optimizer:
    """Base class. Subclasses implement ``_step_cpu_param`` and ``_step_fused``."""

    KIND = "?"

    def __init__(self, params, lr: float, **hyper):
        groups = self._normalise_groups(params, lr, hyper)
        self.groups: List[ParamGroup] = groups
        self.state: Dict[int, dict] = {}
        self.fused = True
        self.gscale_t: Optional[torch.Tensor] = None  # optional device-side grad scale

    @staticmethod
    def _normalise_groups(params, lr, hyper) -> List[ParamGroup]:
        params = list(params)
        if params and isinstance(params[0], dict):
            out = []
            for g in params:
                g = dict(g)
                ps = [p for p in g.pop("params")]
                out.append(ParamGroup(ps, g.pop("lr", lr), **{**hyper, **g}))
            return out
        return [ParamGroup([p for p in params], lr, **hyper)]

    # ---------------------------------------------------------------- params
    @property
    def params(self) -> List[torch.Tensor]:
        return [p for g in self.groups for p in g.params]

    def lr(self) -> float:
        return self.groups[0].lr

    def set_lr(self, lr: float) -> None:
        for g in self.groups:
            g.lr = float(lr)

    def set_group_lr(self, group: int, lr: float) -> None:
        self.groups[group].lr = float(lr)

    def scale_lr(self, factor: float) -> None:
        for g in self.groups:
            g.lr *= factor

    def zero_grad(self, set_to_none: bool = True) -> None:
        for g in self.groups:
            if g.arena is not None and g.arena.is_bound():
                g.arena.zero_grad()
                continue
            for p in g.params:
                if set_to_none:
                    p.grad = None
                elif p.grad is not None:
                    p.grad.zero_()

    def reset_state(self) -> None:
        self.state.clear()
        for g in self.groups:
            self._reset_group_state(g)

    def _reset_group_state(self, g: ParamGroup) -> None:
        if g.step_t is not None:
            g.step_t.zero_()

    # ---------------------------------------------------------------- step
    def _fusable(self, g: ParamGroup) -> bool:
        ps = [p for p in g.params if p.requires_grad]
        return (self.fused and len(ps) == len(g.params) and len(ps) > 0
                and all(p.is_cuda and p.dtype == torch.float32 for p in ps)
                and type(self)._step_fused is not Optimizer._step_fused)

    def ensure_arena(self, g: ParamGroup) -> ParamArena:
        if g.arena is None or not g.arena.is_bound():
            existing = arena_of(g.params)
            g.arena = existing if existing is not None else ParamArena(g.params)
            self._init_fused_state(g)
        return g.arena

    def adopt_arena(self, g: ParamGroup, arena: ParamArena) -> None:
        """Make ``arena`` (e.g. parameters moved into a peer-shared region)
        the group's fused storage. The fused optimizer state is created on the
        group's first arena and kept across later moves (same element order)."""
        first = g.arena is None
        g.arena = arena
        if first:
            self._init_fused_state(g)

    def _device_scalars(self, g: ParamGroup) -> None:
        dev = g.params[0].device
        if g.lr_t is None:
            g.lr_t = torch.full((), g.lr, device=dev, dtype=torch.float32)
            g.lr_t_val = g.lr
            g.step_t = torch.zeros((), device=dev, dtype=torch.float32)
        elif g.lr_t_val != g.lr:
            g.lr_t.fill_(g.lr)
            g.lr_t_val = g.lr

    @torch.no_grad()
    def step(self) -> None:
        for g in self.groups:
            if self._fusable(g):
                self.ensure_arena(g)
                self._device_scalars(g)
                self._step_fused(g)
            else:
                self._step_cpu(g)

    def _step_cpu(self, g: ParamGroup) -> None:
        for p in g.params:
            if p.grad is None:
                continue
            st = self.state.setdefault(id(p), {})
            self._step_cpu_param(g, p, p.grad, st)

    # subclass API
    def _init_fused_state(self, g: ParamGroup) -> None:
        pass

    def _step_fused(self, g: ParamGroup) -> None:  # pragma: no cover - overridden
        raise NotImplementedError

    def _step_cpu_param(self, g, p, grad, st) -> None:  # pragma: no cover - overridden
        raise NotImplementedError

    # ---------------------------------------------------------------- state files
    def save_state(self, w) -> None:
        raise NotImplementedError(f"{self.KIND} does not implement state save")

    def load_state(self, r) -> None:
        raise NotImplementedError(f"{self.KIND} does not implement state load")

    def save_state_file(self, path: str) -> None:
        buf = io.BytesIO()
        buf.write(STATE_MAGIC)
        buf.write(struct.pack("<II", STATE_VERSION, KIND_TAGS[self.KIND]))
        self.save_state(buf)
        _atomic_write(path, buf.getvalue())

    save_state_to = save_state_file

    def load_state_file(self, path: str) -> None:
        with _open_read(path) as f:
            r = io.BytesIO(f.read())
        magic = r.read(4)
        if magic != STATE_MAGIC:
            raise ValueError(f"{path}: not a flodl optimizer state file (missing FDLO header)")
        version, tag = struct.unpack("<II", r.read(8))
        if version > STATE_VERSION:
            raise ValueError(f"{path}: state file version {version} is newer than supported")
        if tag != KIND_TAGS[self.KIND]:
            name = {v: k for k, v in KIND_TAGS.items()}.get(tag, "?")
            raise ValueError(f"{path}: state file was written by {name} but is being loaded into {self.KIND}")
        self.load_state(r)

    # group table: count(u32) | (lr f64, start i64, end i64)*
    def _write_groups(self, w) -> None:
        if len(self.groups) == 1:
            w.write(struct.pack("<I", 0))
            return
        w.write(struct.pack("<I", len(self.groups)))
        start = 0
        for g in self.groups:
            end = start + len(g.params)
            w.write(struct.pack("<dqq", g.lr, start, end))
            start = end

    def _read_groups(self, r) -> None:
        (ng,) = struct.unpack("<I", r.read(4))
        n = len(self.params)
        expected = 0
        lrs = []
        for i in range(ng):
            lr, start, end = struct.unpack("<dqq", r.read(24))
            if start != expected or end < start or end > n:
                raise ValueError(f"corrupt optimizer state: group {i} range {start}..{end}")
            expected = end
            lrs.append(lr)
        if ng and expected != n:
            raise ValueError(f"corrupt optimizer state: groups cover 0..{expected} of {n}")
        if ng == len(self.groups):
            for g, lr in zip(self.groups, lrs):
                g.lr = lr


# ====================================================================== SGD
class SGD(Optimizer):
    """SGD with momentum / dampening / Nesterov / weight decay."""

    KIND = "SGD"

    def __init__(self, params, lr: float, momentum: float = 0.0, weight_decay: float = 0.0,
                 dampening: float = 0.0, nesterov: bool = False):
        super().__init__(params, lr, momentum=momentum, weight_decay=weight_decay,
                         dampening=dampening, nesterov=nesterov)

    def _init_fused_state(self, g):
        if g.hyper["momentum"] != 0.0:
            g.buf = torch.zeros(g.arena.numel, device=g.arena.device)
        else:
            g.buf = None
        g.first_t = torch.ones((), device=g.arena.device)

    def _reset_group_state(self, g):
        super()._reset_group_state(g)
        if getattr(g, "buf", None) is not None:
            g.buf.zero_()
            g.first_t.fill_(1.0)

    def _step_fused(self, g):
        h = g.hyper
        a = g.arena
        cuda_ext().sgd(a.data, a.grad, g.buf, a.shadow, g.lr_t, self.gscale_t, g.first_t,
                       h["momentum"], h["dampening"], h["weight_decay"], h["nesterov"], False)
        if g.buf is not None:
            g.first_t.zero_()

    def _step_cpu_param(self, g, p, grad, st):
        h = g.hyper
        d = grad + h["weight_decay"] * p if h["weight_decay"] else grad.clone()
        if h["momentum"]:
            buf = st.get("momentum_buffer")
            if buf is None:
                buf = d.clone()
            else:
                buf.mul_(h["momentum"]).add_(d, alpha=1 - h["dampening"])
            st["momentum_buffer"] = buf
            d = d + h["momentum"] * buf if h["nesterov"] else buf
        p.add_(d, alpha=-g.lr)

    def velocity(self, p):
        g = next(gr for gr in self.groups if any(q is p for q in gr.params))
        if g.arena is not None and getattr(g, "buf", None) is not None:
            i = next(i for i, q in enumerate(g.arena.params) if q is p)
            return g.arena.view(g.buf, i)
        return self.state.get(id(p), {}).get("momentum_buffer")

    def save_state(self, w):
        ps = self.params
        w.write(struct.pack("<Id", len(ps), self.lr()))
        w.write(struct.pack("<d", self.groups[0].hyper["weight_decay"]))
        for p in ps:
            write_tensor_state(w, self.velocity(p))
        self._write_groups(w)

    def load_state(self, r):
        (n,) = struct.unpack("<I", r.read(4))
        if n != len(self.params):
            raise ValueError(f"SGD: param count mismatch: checkpoint={n} optimizer={len(self.params)}")
        (lr,) = struct.unpack("<d", r.read(8))
        (wd,) = struct.unpack("<d", r.read(8))
        self.set_lr(lr)
        for g in self.groups:
            g.hyper["weight_decay"] = wd
        for p in self.params:
            v = read_tensor_state(r, p.device)
            g = next(gr for gr in self.groups if any(q is p for q in gr.params))
            if g.arena is not None and getattr(g, "buf", None) is not None and v is not None:
                i = next(i for i, q in enumerate(g.arena.params) if q is p)
                g.arena.view(g.buf, i).copy_(v)
                g.first_t.zero_()
            elif v is not None:
                self.state.setdefault(id(p), {})["momentum_buffer"] = v
        self._read_groups(r)


# ====================================================================== Adam / AdamW
class Adam(Optimizer):
    """Adam (Kingma & Ba 2015); L2 weight decay folded into the gradient."""

    KIND = "Adam"
    DECOUPLED = False

    def __init__(self, params, lr: float = 1e-3, beta1: float = 0.9, beta2: float = 0.999,
                 eps: float = 1e-8, weight_decay: float = 0.0, betas=None):
        if betas is not None:
            beta1, beta2 = betas
        super().__init__(params, lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay)

    def _init_fused_state(self, g):
        a = g.arena
        g.m = torch.zeros(a.numel, device=a.device)
        g.v = torch.zeros(a.numel, device=a.device)
        # adopt CPU-path moments accumulated before the arena existed
        for i, p in enumerate(a.params):
            st = self.state.get(id(p))
            if st and "m" in st:
                a.view(g.m, i).copy_(st["m"])
                a.view(g.v, i).copy_(st["v"])

    def _reset_group_state(self, g):
        super()._reset_group_state(g)
        if getattr(g, "m", None) is not None:
            g.m.zero_()
            g.v.zero_()

    def _step_fused(self, g):
        h = g.hyper
        a = g.arena
        C = cuda_ext()
        C.add_scalar(g.step_t, 1.0)
        C.adamw(a.data, a.grad, g.m, g.v, a.shadow, g.lr_t, g.step_t, self.gscale_t, h["beta1"],
                h["beta2"], h["eps"], h["weight_decay"], self.DECOUPLED, False)

    def _step_cpu_param(self, g, p, grad, st):
        h = g.hyper
        b1, b2, eps, wd = h["beta1"], h["beta2"], h["eps"], h["weight_decay"]
        if "m" not in st:
            st["m"] = torch.zeros_like(p)
            st["v"] = torch.zeros_like(p)
            st["step"] = 0
        st["step"] += 1
        t = st["step"]
        if self.DECOUPLED:
            p.mul_(1 - g.lr * wd)
        elif wd:
            grad = grad + wd * p
        st["m"].mul_(b1).add_(grad, alpha=1 - b1)
        st["v"].mul_(b2).addcmul_(grad, grad, value=1 - b2)
        bc1 = 1 - b1 ** t
        bc2 = 1 - b2 ** t
        denom = (st["v"].sqrt() / math.sqrt(bc2)).add_(eps)
        p.addcdiv_(st["m"], denom, value=-g.lr / bc1)

    def _moments(self, p):
        for g in self.groups:
            if g.arena is not None and getattr(g, "m", None) is not None:
                for i, q in enumerate(g.arena.params):
                    if q is p:
                        step = int(g.step_t.item()) if g.step_t is not None else 0
                        return g.arena.view(g.m, i), g.arena.view(g.v, i), step
        st = self.state.get(id(p), {})
        return st.get("m"), st.get("v"), st.get("step", 0)

    def save_state(self, w):
        ps = self.params
        w.write(struct.pack("<Id", len(ps), self.lr()))
        for p in ps:
            m, v, step = self._moments(p)
            write_tensor_state(w, m)
            write_tensor_state(w, v)
            w.write(struct.pack("<q", step))
        self._write_groups(w)

    def load_state(self, r):
        (n,) = struct.unpack("<I", r.read(4))
        if n != len(self.params):
            raise ValueError(f"{self.KIND}: param count mismatch: checkpoint={n} optimizer={len(self.params)}")
        (lr,) = struct.unpack("<d", r.read(8))
        self.set_lr(lr)
        for p in self.params:
            m = read_tensor_state(r, p.device)
            v = read_tensor_state(r, p.device)
            (step,) = struct.unpack("<q", r.read(8))
            placed = False
            for g in self.groups:
                if g.arena is not None and getattr(g, "m", None) is not None:
                    for i, q in enumerate(g.arena.params):
                        if q is p:
                            if m is not None:
                                g.arena.view(g.m, i).copy_(m)
                                g.arena.view(g.v, i).copy_(v)
                            g.step_t.fill_(float(step))
                            placed = True
            if not placed and m is not None:
                self.state[id(p)] = {"m": m, "v": v, "step": step}
        self._read_groups(r)


class AdamW(Adam):
    """AdamW: Adam with decoupled weight decay (Loshchilov & Hutter 2017).
    Positional signature follows floDl: ``AdamW(params, lr, weight_decay)``."""

    KIND = "AdamW"
    DECOUPLED = True

    def __init__(self, params, lr: float = 1e-3, weight_decay: float = 0.01, beta1: float = 0.9,
                 beta2: float = 0.999, eps: float = 1e-8, betas=None):
        super().__init__(params, lr, beta1, beta2, eps, weight_decay, betas)


# ====================================================================== others (ATen math)
class RMSprop(Optimizer):
    KIND = "RMSprop"

    def __init__(self, params, lr: float = 1e-2, alpha: float = 0.99, eps: float = 1e-8,
                 weight_decay: float = 0.0, momentum: float = 0.0, centered: bool = False):
        super().__init__(params, lr, alpha=alpha, eps=eps, weight_decay=weight_decay,
                         momentum=momentum, centered=centered)
        self.fused = False

    def _step_cpu_param(self, g, p, grad, st):
        h = g.hyper
        if h["weight_decay"]:
            grad = grad + h["weight_decay"] * p
        sq = st.setdefault("square_avg", torch.zeros_like(p))
        sq.mul_(h["alpha"]).addcmul_(grad, grad, value=1 - h["alpha"])
        if h["centered"]:
            ga = st.setdefault("grad_avg", torch.zeros_like(p))
            ga.mul_(h["alpha"]).add_(grad, alpha=1 - h["alpha"])
            avg = (sq - ga * ga).sqrt_().add_(h["eps"])
        else:
            avg = sq.sqrt().add_(h["eps"])
        if h["momentum"] > 0:
            buf = st.setdefault("momentum_buffer", torch.zeros_like(p))
            buf.mul_(h["momentum"]).addcdiv_(grad, avg)
            p.add_(buf, alpha=-g.lr)
        else:
            p.addcdiv_(grad, avg, value=-g.lr)

    def save_state(self, w):
        ps = self.params
        w.write(struct.pack("<Id", len(ps), self.lr()))
        for p in ps:
            st = self.state.get(id(p), {})
            write_tensor_state(w, st.get("square_avg"))
            write_tensor_state(w, st.get("momentum_buffer"))
            write_tensor_state(w, st.get("grad_avg"))
        self._write_groups(w)

    def load_state(self, r):
        (n,) = struct.unpack("<I", r.read(4))
        (lr,) = struct.unpack("<d", r.read(8))
        self.set_lr(lr)
        for p in self.params:
            st = {}
            for k in ("square_avg", "momentum_buffer", "grad_avg"):
                t = read_tensor_state(r, p.device)
                if t is not None:
                    st[k] = t
            self.state[id(p)] = st
        self._read_groups(r)


class Adagrad(Optimizer):
    KIND = "Adagrad"

    def __init__(self, params, lr: float = 1e-2, lr_decay: float = 0.0, weight_decay: float = 0.0,
                 eps: float = 1e-10, initial_accumulator_value: float = 0.0):
        super().__init__(params, lr, lr_decay=lr_decay, weight_decay=weight_decay, eps=eps,
                         init_acc=initial_accumulator_value)
        self.fused = False

    def _step_cpu_param(self, g, p, grad, st):
        h = g.hyper
        st["step"] = st.get("step", 0) + 1
        if h["weight_decay"]:
            grad = grad + h["weight_decay"] * p
        s = st.setdefault("sum", torch.full_like(p, h["init_acc"]))
        clr = g.lr / (1 + (st["step"] - 1) * h["lr_decay"])
        s.addcmul_(grad, grad, value=1.0)
        p.addcdiv_(grad, s.sqrt().add_(h["eps"]), value=-clr)

    def save_state(self, w):
        ps = self.params
        w.write(struct.pack("<Id", len(ps), self.lr()))
        for p in ps:
            st = self.state.get(id(p), {})
            write_tensor_state(w, st.get("sum"))
            w.write(struct.pack("<q", st.get("step", 0)))
        self._write_groups(w)

    def load_state(self, r):
        (n,) = struct.unpack("<I", r.read(4))
        (lr,) = struct.unpack("<d", r.read(8))
        self.set_lr(lr)
        for p in self.params:
            s = read_tensor_state(r, p.device)
            (step,) = struct.unpack("<q", r.read(8))
            self.state[id(p)] = {"step": step, **({"sum": s} if s is not None else {})}
        self._read_groups(r)


class RAdam(Adam):
    """Rectified Adam (Liu et al. 2020)."""

    KIND = "RAdam"

    def __init__(self, params, lr: float = 1e-3, beta1: float = 0.9, beta2: float = 0.999,
                 eps: float = 1e-8, weight_decay: float = 0.0):
        super().__init__(params, lr, beta1, beta2, eps, weight_decay)
        self.fused = False

    def _step_cpu_param(self, g, p, grad, st):
        h = g.hyper
        b1, b2 = h["beta1"], h["beta2"]
        if h["weight_decay"]:
            grad = grad + h["weight_decay"] * p
        if "m" not in st:
            st.update(m=torch.zeros_like(p), v=torch.zeros_like(p), step=0)
        st["step"] += 1
        t = st["step"]
        st["m"].mul_(b1).add_(grad, alpha=1 - b1)
        st["v"].mul_(b2).addcmul_(grad, grad, value=1 - b2)
        mhat = st["m"] / (1 - b1 ** t)
        rho_inf = 2 / (1 - b2) - 1
        rho_t = rho_inf - 2 * t * b2 ** t / (1 - b2 ** t)
        if rho_t > 5:
            vhat = (st["v"] / (1 - b2 ** t)).sqrt_().add_(h["eps"])
            r = math.sqrt((rho_t - 4) * (rho_t - 2) * rho_inf / ((rho_inf - 4) * (rho_inf - 2) * rho_t))
            p.addcdiv_(mhat, vhat, value=-g.lr * r)
        else:
            p.add_(mhat, alpha=-g.lr)


class NAdam(Adam):
    """Adam with Nesterov momentum (Dozat 2016), PyTorch's momentum-decay schedule."""

    KIND = "NAdam"

    def __init__(self, params, lr: float = 2e-3, beta1: float = 0.9, beta2: float = 0.999,
                 eps: float = 1e-8, weight_decay: float = 0.0, momentum_decay: float = 4e-3):
        super().__init__(params, lr, beta1, beta2, eps, weight_decay)
        for g in self.groups:
            g.hyper["momentum_decay"] = momentum_decay
        self.fused = False

    def _step_cpu_param(self, g, p, grad, st):
        h = g.hyper
        b1, b2 = h["beta1"], h["beta2"]
        if h["weight_decay"]:
            grad = grad + h["weight_decay"] * p
        if "m" not in st:
            st.update(m=torch.zeros_like(p), v=torch.zeros_like(p), step=0, mu_product=1.0)
        st["step"] += 1
        t = st["step"]
        mu = b1 * (1 - 0.5 * 0.96 ** (t * h["momentum_decay"]))
        mu_next = b1 * (1 - 0.5 * 0.96 ** ((t + 1) * h["momentum_decay"]))
        st["mu_product"] *= mu
        mp = st["mu_product"]
        st["m"].mul_(b1).add_(grad, alpha=1 - b1)
        st["v"].mul_(b2).addcmul_(grad, grad, value=1 - b2)
        denom = (st["v"] / (1 - b2 ** t)).sqrt_().add_(h["eps"])
        p.addcdiv_(grad, denom, value=-g.lr * (1 - mu) / (1 - mp))
        p.addcdiv_(st["m"], denom, value=-g.lr * mu_next / (1 - mp * mu_next))


def migrate_optim_state_file(src: str, dst: str, kind: str) -> None:
    """Prefix a pre-header (headerless) state file with the FDLO header."""
    with _open_read(src) as f:
        data = f.read()
    if data[:4] == STATE_MAGIC:
        raise ValueError(f"{src}: already has an FDLO header")
    payload = STATE_MAGIC + struct.pack("<II", STATE_VERSION, KIND_TAGS[kind]) + data
    _atomic_write(dst, payload)
