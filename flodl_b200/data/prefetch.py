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
    def __init__(self, host: List[torch.Tensor], order: torch.Tensor, bs: int, nb: int, device,
                 depth: int = 2):
        self.host = host
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
                rows = [t.index_select(0, idx) for t in self.host]
                if self.cuda:
                    pinned = [r.pin_memory() for r in rows]
                    with torch.cuda.stream(self.stream):
                        dev = [p.to(self.device, non_blocking=True) for p in pinned]
                        ev = torch.cuda.Event()
                        ev.record(self.stream)
                    self.q.put((dev, ev, pinned))
                else:
                    self.q.put((rows, None, None))
        except BaseException as e:  # surfaced to the consumer
            self.q.put(e)
        self.q.put(None)

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
