"""CPU averaging backend: controller, client, heartbeats and dead-rank detection.

Reference roles: the CPU-reduce controller (flodl/src/distributed/controller/
mod.rs:333, round_frame.rs:517-540), its client (cpu_reduce.rs:202-804), and
the coordinator's dead-rank detection (cluster_coordinator/dead_ranks.rs:27-100).

Protocol (signed frames from the native wire codec, one TCP connection per
rank):

    HELLO(rank)                       rank -> controller
    ROUND(round, mass, dtype, bytes)  rank -> controller: payload = params * mass
    CONSENSUS(round, bytes)           controller -> rank: sum(payloads) / sum(mass)
    HEARTBEAT(rank)                   rank -> controller, every ``heartbeat_s``
    DEAD(rank)                        controller -> ranks when a heartbeat is stale
    BCAST(round, rank, root flag, dtype, bytes)
                                      rank -> controller: initial-state broadcast;
                                      the root's bytes go to every rank once all
                                      alive ranks asked (the others send none)
    HOSTFRAME(round, mass, dtype, ranks, bytes)
                                      relay -> controller: the folded sum of a
                                      host's ranks (flodl_b200.parallel.relay)

One connection may carry several ranks (a per-host relay): every HELLO on it
registers one more rank, a HEARTBEAT or BYE with a rank payload speaks for
that rank only, and a DEAD from a relay reports a local rank that exited.

A round completes when every live rank contributed; a rank whose heartbeat is
older than ``heartbeat_timeout`` is declared dead, dropped from membership
(membership only shrinks) and the round proceeds without it. Payloads travel
as f32 or bf16 (halving the wire bytes); the reduction sums in f32 with the
mass folded in by the sender and divides once by the accepted mass.
"""
from __future__ import annotations

import socket
import struct
import threading
import time
from typing import Dict, List, Optional, Tuple

import torch

from .._ext import native

MAGIC = 0x464C4443  # "FLDC"
K_HELLO, K_ROUND, K_CONSENSUS, K_HEARTBEAT, K_DEAD, K_BYE, K_HOSTFRAME = 1, 2, 3, 4, 5, 6, 7
K_BCAST = 8
DT_F32, DT_BF16 = 0, 1
MAX_FRAME = 1 << 34


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(min(n - len(buf), 1 << 20))
        if not chunk:
            raise ConnectionError("peer closed")
        buf += chunk
    return bytes(buf)


def send_frame(sock, key: bytes, kind: int, seq: int, payload: bytes, lock=None,
               magic: int = MAGIC) -> None:
    f = native().encode_frame(magic, kind, seq, payload, key)
    if lock:
        with lock:
            sock.sendall(f)
    else:
        sock.sendall(f)


def recv_frame(sock, key: bytes, magic: int = MAGIC,
               max_frame: int = MAX_FRAME) -> Tuple[int, int, bytes]:
    """Read one signed frame; raises ConnectionError on a wrong channel magic,
    an oversized frame or a bad signature."""
    N = native()
    hdr = _recv_exact(sock, N.WIRE_HEADER_BYTES)
    got, kind, flags, seq, ln = N.peek_header(hdr)
    if got != magic:
        raise ConnectionError("bad frame magic")
    if ln > max_frame:
        raise ConnectionError("frame exceeds ceiling")
    rest = _recv_exact(sock, ln + 8)
    try:
        _m, kind, _f, seq, payload = N.decode_frame(hdr + rest, key, max_frame)
    except Exception as e:  # signature or format failure
        raise ConnectionError(f"rejected frame: {e}") from e
    return kind, seq, payload


def encode_tensor(t: torch.Tensor, bf16: bool) -> Tuple[int, bytes]:
    t = t.detach().float().contiguous().cpu()
    if bf16:
        return DT_BF16, native().f32_to_bf16_bits(t).numpy().tobytes()
    return DT_F32, t.numpy().tobytes()


def decode_tensor(dt: int, raw: bytes) -> torch.Tensor:
    if dt == DT_BF16:
        bits = torch.frombuffer(bytearray(raw), dtype=torch.int16)
        return native().bf16_bits_to_f32(bits)
    return torch.frombuffer(bytearray(raw), dtype=torch.float32).clone()


class CpuReduceController:
    """Accepts rank connections, runs reduce rounds, tracks heartbeats."""

    def __init__(self, world: int, key: bytes, host: str = "127.0.0.1", port: Optional[int] = 0,
                 heartbeat_timeout: float = 30.0):
        """``port=None`` binds nothing: connections arrive through :meth:`adopt`
        (the single-port mux of :mod:`flodl_b200.parallel.portmux`)."""
        self.world = world
        self.key = key
        self.hb_timeout = heartbeat_timeout
        self.srv = None
        self.port = None
        if port is not None:
            self.srv = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
            self.srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            self.srv.bind((host, port))
            self.srv.listen(world + 8)
            self.port = self.srv.getsockname()[1]
        self.conns: Dict[int, socket.socket] = {}
        self.send_locks: Dict[int, threading.Lock] = {}
        self.alive = set(range(world))
        self.dead: List[int] = []
        self.last_hb: Dict[int, float] = {}
        self.pending: Dict[int, Dict[int, Tuple[Optional[torch.Tensor], float]]] = {}
        self.host_parts: Dict[int, List[Tuple[torch.Tensor, float]]] = {}
        self.bcasts: Dict[int, dict] = {}  # rnd -> {"ranks": set, "payload": bytes | None}
        self.lock = threading.Lock()
        self.cv = threading.Condition(self.lock)
        self.rejected = 0
        self.frames_in = 0        # data frames received (ROUND + HOSTFRAME)
        self.bytes_in = 0         # their payload bytes
        self._stop = threading.Event()
        self.rounds_done = 0
        if self.srv is not None:
            threading.Thread(target=self._accept_loop, daemon=True).start()
        threading.Thread(target=self._watchdog, daemon=True).start()

    # ------------------------------------------------------------ plumbing
    def _accept_loop(self):
        while not self._stop.is_set():
            try:
                c, _ = self.srv.accept()
            except OSError:
                return
            self.adopt(c)

    def adopt(self, c: socket.socket) -> None:
        """Serve a connection accepted elsewhere (its first bytes unread)."""
        threading.Thread(target=self._serve, args=(c,), daemon=True).start()

    def _register(self, c: socket.socket, rank: int, lock: threading.Lock) -> None:
        with self.lock:
            self.conns[rank] = c
            self.send_locks[rank] = lock
            self.last_hb[rank] = time.time()

    def _declare_dead(self, rank: int) -> None:
        with self.cv:
            if rank not in self.alive:
                return
            self.alive.discard(rank)
            self.dead.append(rank)
            for rnd in list(self.pending):
                self._maybe_finish(rnd)
        self._broadcast(K_DEAD, 0, struct.pack("<i", rank))

    def _serve(self, c: socket.socket):
        mine: List[int] = []
        lock = threading.Lock()
        try:
            kind, _, payload = recv_frame(c, self.key)
            if kind != K_HELLO:
                raise ConnectionError("expected HELLO")
            (rank,) = struct.unpack("<i", payload)
            mine.append(rank)
            self._register(c, rank, lock)
            while not self._stop.is_set():
                kind, seq, payload = recv_frame(c, self.key)
                if kind == K_HEARTBEAT:
                    now = time.time()
                    who = struct.unpack("<i", payload) if len(payload) == 4 else mine
                    with self.lock:
                        for r in who:
                            self.last_hb[r] = now
                elif kind == K_ROUND:
                    rnd, mass, dt = struct.unpack("<qdi", payload[:20])
                    t = decode_tensor(dt, payload[20:])
                    with self.cv:
                        self.frames_in += 1
                        self.bytes_in += len(payload)
                        self.last_hb[mine[0]] = time.time()
                        self.pending.setdefault(rnd, {})[mine[0]] = (t, mass)
                        self._maybe_finish(rnd)
                elif kind == K_HOSTFRAME:
                    rnd, mass, dt, nr = struct.unpack("<qdii", payload[:24])
                    ranks = struct.unpack(f"<{nr}i", payload[24:24 + 4 * nr])
                    t = decode_tensor(dt, payload[24 + 4 * nr:])
                    with self.cv:
                        self.frames_in += 1
                        self.bytes_in += len(payload)
                        now = time.time()
                        got = self.pending.setdefault(rnd, {})
                        for r in ranks:
                            got[r] = (None, 0.0)
                            self.last_hb[r] = now
                        self.host_parts.setdefault(rnd, []).append((t, mass))
                        self._maybe_finish(rnd)
                elif kind == K_BCAST:  # the sender's rank rides in the payload (relays)
                    rnd, who, is_root, dt = struct.unpack("<qiii", payload[:20])
                    with self.cv:
                        b = self.bcasts.setdefault(rnd, {"ranks": set(), "payload": None})
                        b["ranks"].add(who)
                        if is_root:
                            b["payload"] = struct.pack("<qi", rnd, dt) + payload[20:]
                        self._maybe_bcast(rnd)
                elif kind == K_HELLO:  # relay: one more local rank on this connection
                    (r,) = struct.unpack("<i", payload)
                    mine.append(r)
                    self._register(c, r, lock)
                elif kind == K_DEAD:  # relay: a local rank exited
                    (r,) = struct.unpack("<i", payload)
                    self._declare_dead(r)
                elif kind == K_BYE:
                    if len(payload) == 4:
                        (r,) = struct.unpack("<i", payload)
                        if r in mine:
                            mine.remove(r)
                        if mine:
                            continue
                    break
        except Exception:
            with self.lock:
                self.rejected += 1
        finally:
            try:
                c.close()
            except OSError:
                pass

    def _watchdog(self):
        while not self._stop.is_set():
            time.sleep(min(0.2, self.hb_timeout / 4))
            now = time.time()
            newly = []
            with self.cv:
                for r in list(self.alive):
                    t = self.last_hb.get(r)
                    if t is not None and now - t > self.hb_timeout:
                        self.alive.discard(r)
                        self.dead.append(r)
                        newly.append(r)
                for rnd in list(self.pending):
                    self._maybe_finish(rnd)
            for r in newly:
                self._broadcast(K_DEAD, 0, struct.pack("<i", r))

    def _broadcast(self, kind, seq, payload, ranks=None):
        sent = set()  # a relay's connection carries several ranks: send once
        for r in list(ranks if ranks is not None else self.alive):
            c = self.conns.get(r)
            if c is None or id(c) in sent:
                continue
            sent.add(id(c))
            try:
                send_frame(c, self.key, kind, seq, payload, self.send_locks[r])
            except OSError:
                pass

    def _maybe_bcast(self, rnd: int):
        b = self.bcasts.get(rnd)
        if b is None or b["payload"] is None or not self.alive.issubset(b["ranks"]):
            return
        del self.bcasts[rnd]
        self._broadcast(K_CONSENSUS, rnd % (1 << 64), b["payload"], sorted(self.alive))

    def _maybe_finish(self, rnd: int):
        got = self.pending.get(rnd, {})
        if not self.alive or not self.alive.issubset(got.keys()):
            return
        contribs = [got[r] for r in sorted(self.alive) if got[r][0] is not None]
        contribs += self.host_parts.pop(rnd, [])
        out = native().reduce_scaled([t for t, _ in contribs], [m for _, m in contribs])
        dt, raw = DT_F32, out.numpy().tobytes()
        payload = struct.pack("<qi", rnd, dt) + raw
        ranks = sorted(got.keys() & self.alive)
        del self.pending[rnd]
        self.rounds_done += 1
        self._broadcast(K_CONSENSUS, rnd % (1 << 64), payload, ranks)

    def close(self):
        self._stop.set()
        try:
            if self.srv is not None:
                self.srv.close()
        except OSError:
            pass
        for c in list(self.conns.values()):
            try:
                c.close()
            except OSError:
                pass


class CpuReduceClient:
    """Rank side: ``all_reduce_scaled(params, mass)`` returns the mass-weighted
    consensus; a background thread sends heartbeats."""

    def __init__(self, rank: int, host: str, port: int, key: bytes, heartbeat_s: float = 1.0,
                 bf16_wire: bool = False, timeout: float = 120.0):
        self.rank = rank
        self.key = key
        self.bf16 = bf16_wire
        self.sock = socket.create_connection((host, port), timeout=timeout)
        self.sock.settimeout(timeout)
        self.lock = threading.Lock()
        send_frame(self.sock, key, K_HELLO, 0, struct.pack("<i", rank), self.lock)
        self.dead: List[int] = []
        self._inbox: Dict[int, torch.Tensor] = {}
        self._cv = threading.Condition()
        self._stop = threading.Event()
        self.heartbeat_s = heartbeat_s
        self._hb = threading.Thread(target=self._heartbeat, daemon=True)
        self._hb.start()
        threading.Thread(target=self._reader, daemon=True).start()

    def _heartbeat(self):
        while not self._stop.wait(self.heartbeat_s):
            try:
                send_frame(self.sock, self.key, K_HEARTBEAT, 0, b"", self.lock)
            except OSError:
                return

    def stop_heartbeat(self):
        """Test hook: silence this rank's heartbeat (simulates a hung rank)."""
        self._stop.set()

    def _reader(self):
        try:
            while True:
                kind, seq, payload = recv_frame(self.sock, self.key)
                if kind == K_CONSENSUS:
                    rnd, dt = struct.unpack("<qi", payload[:12])
                    t = decode_tensor(dt, payload[12:])
                    with self._cv:
                        self._inbox[rnd] = t
                        self._cv.notify_all()
                elif kind == K_DEAD:
                    (r,) = struct.unpack("<i", payload)
                    with self._cv:
                        self.dead.append(r)
                        self._cv.notify_all()
        except Exception:
            with self._cv:
                self._cv.notify_all()

    def all_reduce_scaled(self, t: torch.Tensor, mass: float, rnd: int,
                          timeout: float = 120.0) -> torch.Tensor:
        dt, raw = encode_tensor(t.detach().float() * mass, self.bf16)
        payload = struct.pack("<qdi", rnd, float(mass), dt) + raw
        send_frame(self.sock, self.key, K_ROUND, rnd % (1 << 64), payload, self.lock)
        deadline = time.time() + timeout
        with self._cv:
            while rnd not in self._inbox:
                left = deadline - time.time()
                if left <= 0:
                    raise TimeoutError(f"rank {self.rank}: reduce round {rnd} timed out")
                self._cv.wait(left)
            out = self._inbox.pop(rnd)
        return out.reshape(t.shape).to(t.device, t.dtype)

    def broadcast_from_root(self, t: torch.Tensor, root: int, rnd: int,
                            timeout: float = 120.0) -> torch.Tensor:
        """Every rank receives the root's tensor (the initial parameter state);
        non-root ranks send no payload."""
        is_root = self.rank == root
        dt, raw = encode_tensor(t, self.bf16) if is_root else (DT_F32, b"")
        send_frame(self.sock, self.key, K_BCAST, rnd % (1 << 64),
                   struct.pack("<qiii", rnd, self.rank, int(is_root), dt) + raw, self.lock)
        deadline = time.time() + timeout
        with self._cv:
            while rnd not in self._inbox:
                left = deadline - time.time()
                if left <= 0:
                    raise TimeoutError(f"rank {self.rank}: broadcast {rnd} timed out")
                self._cv.wait(left)
            out = self._inbox.pop(rnd)
        return out.reshape(t.shape).to(t.device, t.dtype)

    def close(self):
        self._stop.set()
        try:
            send_frame(self.sock, self.key, K_BYE, 0, b"", self.lock)
        except OSError:
            pass
        try:
            self.sock.close()
        except OSError:
            pass
