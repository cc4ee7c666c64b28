"""Per-host relay: the first fold tier of the CPU averaging reduce.

Reference: flodl/src/distributed/relay/agent.rs (fold station, rank-exit
handling) and relay/mod.rs (one upstream connection per host and channel).

A host runs one :class:`RelayAgent`. Its local ranks dial the relay on
loopback with the unchanged rank protocol (:class:`~.cpu_reduce.CpuReduceClient`);
the relay holds ONE upstream connection to the controller for the whole host:

* each local HELLO and HEARTBEAT is forwarded upstream tagged with its rank;
* ROUND payloads (already scaled by their mass) are folded into the round's
  running f32 sum as they arrive - element-wise sums of payloads and masses,
  never a division (the controller divides exactly once); the deposit that
  completes the round (every locally alive rank merged) ships one HOSTFRAME
  upstream, so uplink bytes scale with hosts, not ranks;
* BCAST (initial-state broadcast) frames are forwarded as they are;
* the controller's CONSENSUS arrives once and is fanned out to the local
  ranks of that round; a DEAD from the controller is forwarded to every local
  rank and drops the rank from the local fold;
* a local rank whose connection ends (EOF or error) is removed from the fold
  (its deposited rounds stay folded) and reported upstream as DEAD, so a
  finished or crashed rank cannot park the host's fold.
"""
from __future__ import annotations

import socket
import struct
import threading
from typing import Dict, List, Optional, Set, Tuple

import torch

from .cpu_reduce import (DT_F32, K_BCAST, K_BYE, K_CONSENSUS, K_DEAD, K_HEARTBEAT, K_HELLO,
                         K_HOSTFRAME, K_ROUND, decode_tensor, recv_frame, send_frame)

RELAY_DATA_LOOPBACK_OFFSET = 4  # loopback port = controller port + 4


class RelayAgent:
    """One per host: loopback listener for local ranks, one upstream link."""

    def __init__(self, upstream: Tuple[str, int], key: bytes, host: str = "127.0.0.1",
                 port: int = 0, timeout: float = 120.0):
        self.key = key
        self.up = socket.create_connection(upstream, timeout=timeout)
        self.up.settimeout(None)
        self.up_lock = threading.Lock()          # single writer of the upstream link
        self.srv = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self.srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.srv.bind((host, port))
        self.srv.listen(64)
        self.port = self.srv.getsockname()[1]
        self.local: Dict[int, socket.socket] = {}
        self.local_locks: Dict[int, threading.Lock] = {}
        self.alive: Set[int] = set()
        self.dead: List[int] = []
        self.rounds: Dict[int, dict] = {}       # rnd -> {"sum", "mass", "ranks"}
        self.frames_up = 0
        self.bytes_up = 0
        self.lock = threading.Lock()
        self._hello_sent = False
        self._stop = threading.Event()
        threading.Thread(target=self._accept_loop, daemon=True).start()
        threading.Thread(target=self._upstream_reader, daemon=True).start()

    # ------------------------------------------------------------ upstream
    def _send_up(self, kind: int, seq: int, payload: bytes) -> None:
        send_frame(self.up, self.key, kind, seq, payload, self.up_lock)

    def _upstream_reader(self) -> None:
        try:
            while not self._stop.is_set():
                kind, seq, payload = recv_frame(self.up, self.key)
                if kind == K_CONSENSUS:
                    with self.lock:
                        targets = [r for r in self.local if r in self.alive]
                    self._fan_out(kind, seq, payload, targets)
                elif kind == K_DEAD:
                    (r,) = struct.unpack("<i", payload)
                    self._drop(r, report=False)
                    with self.lock:
                        targets = list(self.local)
                    self._fan_out(kind, seq, payload, targets)
        except Exception:
            pass
        finally:
            self._stop.set()  # controller gone: tear the host down
            with self.lock:
                socks = list(self.local.values())
            for c in socks:
                try:
                    c.close()
                except OSError:
                    pass

    def _fan_out(self, kind: int, seq: int, payload: bytes, ranks) -> None:
        for r in ranks:
            c, lk = self.local.get(r), self.local_locks.get(r)
            if c is None:
                continue
            try:
                send_frame(c, self.key, kind, seq, payload, lk)
            except OSError:
                pass

    # ------------------------------------------------------------ local ranks
    def _accept_loop(self) -> None:
        while not self._stop.is_set():
            try:
                c, _ = self.srv.accept()
            except OSError:
                return
            threading.Thread(target=self._serve_rank, args=(c,), daemon=True).start()

    def _serve_rank(self, c: socket.socket) -> None:
        rank = None
        try:
            kind, _, payload = recv_frame(c, self.key)
            if kind != K_HELLO:
                raise ConnectionError("expected HELLO")
            (rank,) = struct.unpack("<i", payload)
            with self.lock:
                self.local[rank] = c
                self.local_locks[rank] = threading.Lock()
                self.alive.add(rank)
            self._send_up(K_HELLO, 0, payload)
            while not self._stop.is_set():
                kind, seq, payload = recv_frame(c, self.key)
                if kind == K_HEARTBEAT:
                    self._send_up(K_HEARTBEAT, 0, struct.pack("<i", rank))
                elif kind == K_ROUND:
                    self._deposit(rank, payload)
                elif kind == K_BCAST:  # initial-state broadcast: forwarded (it carries its rank)
                    self._send_up(K_BCAST, seq, payload)
                elif kind == K_BYE:
                    break
        except Exception:
            pass
        finally:
            if rank is not None:
                self._drop(rank, report=True)
            try:
                c.close()
            except OSError:
                pass

    def _deposit(self, rank: int, payload: bytes) -> None:
        rnd, mass, dt = struct.unpack("<qdi", payload[:20])
        t = decode_tensor(dt, payload[20:])
        with self.lock:
            st = self.rounds.setdefault(rnd, {"sum": None, "mass": 0.0, "ranks": []})
            if st["sum"] is None:
                st["sum"] = t
            else:
                st["sum"].add_(t)   # fold: sum only, the controller divides once
            st["mass"] += mass
            st["ranks"].append(rank)
            ready = self._take_ready(rnd)
        if ready is not None:
            self._ship(rnd, *ready)

    def _take_ready(self, rnd: int):
        """Under ``self.lock``: pop the round if every alive local rank deposited."""
        st = self.rounds.get(rnd)
        if st is None or st["sum"] is None or not self.alive.issubset(st["ranks"]):
            return None
        del self.rounds[rnd]
        return st["sum"], st["mass"], st["ranks"]

    def _ship(self, rnd: int, total: torch.Tensor, mass: float, ranks: List[int]) -> None:
        body = total.contiguous().numpy().tobytes()
        payload = (struct.pack("<qdii", rnd, mass, DT_F32, len(ranks))
                   + struct.pack(f"<{len(ranks)}i", *ranks) + body)
        self._send_up(K_HOSTFRAME, rnd % (1 << 64), payload)
        with self.lock:
            self.frames_up += 1
            self.bytes_up += len(payload)

    def _drop(self, rank: int, report: bool) -> None:
        with self.lock:
            if rank not in self.alive:
                return
            self.alive.discard(rank)
            self.dead.append(rank)
            ready = [(rnd, self._take_ready(rnd)) for rnd in list(self.rounds)]
        if report:
            try:
                self._send_up(K_DEAD, 0, struct.pack("<i", rank))
            except OSError:
                pass
        for rnd, r in ready:
            if r is not None:
                self._ship(rnd, *r)

    def close(self) -> None:
        self._stop.set()
        for s in (self.srv, self.up):
            try:
                s.close()
            except OSError:
                pass
        with self.lock:
            socks = list(self.local.values())
        for c in socks:
            try:
                c.close()
            except OSError:
                pass
