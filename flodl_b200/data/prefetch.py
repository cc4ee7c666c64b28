"""Streaming-mode batch prefetcher.

A background thread gathers each batch's rows on the host (``index_select``
into pinned staging buffers) and issues the host-to-device copies on a
dedicated CUDA stream, keeping ``depth`` batches in flight; the consumer waits
on the batch's copy event on its own stream before using it (reference:
streaming mode, flodl/src/data/prefetch.rs, docs/ddp/03-internals.md:233-247).
"""
from __future__ import annotations

import queue
import threading
from typing import List, Optional

import torch


class Prefetcher:
    """``fetch(idx) -> host rows``; with a device sample ``pool`` only the
    pool's misses are uploaded, hits are gathered on the device and the
    uploaded rows are admitted to the pool while it has room."""

    def __init__(self, fetch, order: torch.Tensor, bs: int, nb: int, device,
                 depth: int = 2, pool=None):
        self.fetch = fetch
        self.pool = pool
        self.order = order
        self.bs, self.nb = bs, nb
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.q: "queue.Queue" = queue.Queue(maxsize=max(1, depth))
        self.stream = torch.cuda.Stream(self.device) if self.cuda else None
        self._stop = threading.Event()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        try:
            for i in range(self.nb):
                if self._stop.is_set():
                    break
                idx = self.order[i * self.bs:(i + 1) * self.bs]
                if self.cuda:
                    self.q.put(self._upload(idx))
                else:
                    self.q.put((self.fetch(idx), None, None))
        except BaseException as e:  # surfaced to the consumer
            self.q.put(e)
        self.q.put(None)

    def _upload(self, idx: torch.Tensor):
        pool = self.pool
        if pool is None:
            pinned = [r.pin_memory() for r in self.fetch(idx)]
            with torch.cuda.stream(self.stream):
                dev = [p.to(self.device, non_blocking=True) for p in pinned]
                ev = torch.cuda.Event()
                ev.record(self.stream)
            return dev, ev, pinned
        slots = pool.lookup(idx)
        hit = slots >= 0
        miss_pos = (~hit).nonzero().flatten()
        hit_pos = hit.nonzero().flatten()
        pinned = [r.pin_memory() for r in self.fetch(idx[miss_pos])] if miss_pos.numel() else None
        with torch.cuda.stream(self.stream):
            out = None
            if pinned is not None:
                up = [p.to(self.device, non_blocking=True) for p in pinned]
                out = [torch.empty((idx.numel(), *u.shape[1:]), dtype=u.dtype, device=self.device)
                       for u in up]
                mp = miss_pos.to(self.device, non_blocking=True)
                for o, u in zip(out, up):
                    o.index_copy_(0, mp, u)
                pool.admit(idx[miss_pos], up)
            if hit_pos.numel():
                rows = pool.gather(slots[hit_pos])
                if out is None:
                    out = rows
                else:
                    hp = hit_pos.to(self.device, non_blocking=True)
                    for o, r in zip(out, rows):
                        o.index_copy_(0, hp, r)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        return out, ev, pinned

    def __iter__(self):
        while True:
            item = self.q.get()
            if item is None:
                return
            if isinstance(item, BaseException):
                raise item
            batch, ev, _pinned = item
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
                for b in batch:
                    b.record_stream(torch.cuda.current_stream(self.device))
            yield batch

    def close(self):
        self._stop.set()
        try:
            while True:
                self.q.get_nowait()
        except queue.Empty:
            pass
