"""TCP rendezvous over the signed wire protocol.

Reference: flodl/src/distributed/rendezvous.rs:47-120 (``TcpRendezvous``):
every rank dials one address, says HELLO, receives its ROLE - the first rank
*generates* the communicator's unique id, the others *wait* for it - and
every rank leaves with (rank, world, uid). The server gives up after an idle
period without progress (120 s) and stops accepting after 1024 rejected
connections (bad magic, bad signature, malformed or duplicate HELLO).

Frames are HMAC-signed by the native codec (``flodl_b200._native``) with the
job's shared key; a rank that does not hold the key cannot join.

    HELLO {"rank": r or -1, "host": ..., "info": {...}}     rank -> server
    ROLE  {"rank": r, "world": n, "role": "generate"|"wait", "members": [...]}
    UID   raw bytes (the generator's id)                     generator -> server -> others
    REJECT {"reason": ...}                                   server -> rank
"""
from __future__ import annotations

import json
import os
import queue
import socket
import threading
import time
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence

from .cpu_reduce import recv_frame, send_frame

MAGIC_RDV = 0x464C5256  # "FLRV"
K_HELLO, K_ROLE, K_UID, K_REJECT = 1, 2, 3, 4
IDLE_TIMEOUT_S = 120.0
REJECT_CAP = 1024
MAX_RDV_FRAME = 1 << 20


@dataclass
class RendezvousResult:
    rank: int
    world: int
    uid: bytes
    members: List[dict]


class RendezvousServer:
    """Collects ``world`` HELLOs, assigns ranks (requested ranks are kept,
    the rest fill the gaps in arrival order), then relays rank 0's UID."""

    def __init__(self, world: int, key: bytes, host: str = "127.0.0.1", port: Optional[int] = 0,
                 idle_timeout: float = IDLE_TIMEOUT_S, reject_cap: int = REJECT_CAP,
                 agree_on: Sequence[str] = ("model_sig",)):
        """``port=None`` binds nothing: connections arrive through :meth:`adopt`
        (the single-port mux of :mod:`flodl_b200.parallel.portmux`).
        ``agree_on`` names HELLO ``info`` keys every rank must report equal
        (the model signature by default): a mismatch refuses the formation,
        since ranks training different models would corrupt each other at
        the first collective."""
        self.world, self.key = world, key
        self.agree_on = tuple(agree_on)
        self.idle_timeout, self.reject_cap = idle_timeout, reject_cap
        self.rejected = 0
        self.error: Optional[str] = None
        self.members: List[dict] = []
        self._conns: List[socket.socket] = []
        self._adopted: "queue.Queue[socket.socket]" = queue.Queue()
        self._sock = None
        self.host, self.port = host, None
        if port is not None:
            self._sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
            self._sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            self._sock.bind((host, port))
            self._sock.listen(128)
            self._sock.settimeout(0.2)
            self.host, self.port = self._sock.getsockname()
        self._done = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def start(self) -> "RendezvousServer":
        self._thread.start()
        return self

    def wait(self, timeout: Optional[float] = None) -> bool:
        return self._done.wait(timeout)

    def adopt(self, c: socket.socket) -> None:
        """Take a connection accepted elsewhere (its first bytes unread)."""
        self._adopted.put(c)

    def _accept(self) -> socket.socket:
        if self._sock is None:
            try:
                return self._adopted.get(timeout=0.2)
            except queue.Empty:
                raise socket.timeout() from None
        return self._sock.accept()[0]

    def _reject(self, c: socket.socket, reason: str) -> None:
        self.rejected += 1
        try:
            send_frame(c, self.key, K_REJECT, 0, json.dumps({"reason": reason}).encode(),
                       magic=MAGIC_RDV)
        except OSError:
            pass
        c.close()

    def _run(self) -> None:
        hellos: List[tuple] = []
        last = time.monotonic()
        try:
            while len(hellos) < self.world:
                if time.monotonic() - last > self.idle_timeout:
                    self.error = f"rendezvous idle for {self.idle_timeout:.0f} s with {len(hellos)}/{self.world} ranks"
                    break
                if self.rejected >= self.reject_cap:
                    self.error = f"rendezvous stopped after {self.rejected} rejected connections"
                    break
                try:
                    c = self._accept()
                except socket.timeout:
                    continue
                c.settimeout(10.0)
                try:
                    kind, _, payload = recv_frame(c, self.key, magic=MAGIC_RDV,
                                                  max_frame=MAX_RDV_FRAME)
                    if kind != K_HELLO:
                        raise ConnectionError("expected HELLO")
                    hello = json.loads(payload.decode())
                    want = int(hello.get("rank", -1))
                    if want >= self.world or any(h[0] == want >= 0 for h in hellos):
                        raise ConnectionError(f"rank {want} unavailable")
                except (ConnectionError, OSError, ValueError) as e:
                    self._reject(c, str(e))
                    continue
                hellos.append((want, hello, c))
                last = time.monotonic()
            for k in self.agree_on:
                vals = {json.dumps(h.get("info", {}).get(k)) for _, h, _ in hellos}
                if len(vals) > 1:
                    self.error = f"ranks disagree on {k}: formation refused"
            if self.error:
                for _, _, c in hellos:
                    self._reject(c, self.error)
                return
            # rank assignment: keep requested ranks, fill the rest in arrival order
            taken = {w for w, _, _ in hellos if w >= 0}
            free = iter(r for r in range(self.world) if r not in taken)
            assigned = []
            for w, hello, c in hellos:
                r = w if w >= 0 else next(free)
                assigned.append((r, hello, c))
            assigned.sort(key=lambda t: t[0])
            self.members = [{"rank": r, "host": h.get("host"), "info": h.get("info", {})}
                            for r, h, _ in assigned]
            for r, _, c in assigned:
                role = {"rank": r, "world": self.world,
                        "role": "generate" if r == 0 else "wait", "members": self.members}
                send_frame(c, self.key, K_ROLE, 0, json.dumps(role).encode(), magic=MAGIC_RDV)
            gen = assigned[0][2]
            gen.settimeout(self.idle_timeout)
            kind, _, uid = recv_frame(gen, self.key, magic=MAGIC_RDV, max_frame=MAX_RDV_FRAME)
            if kind != K_UID:
                raise ConnectionError("generator did not send the UID")
            for r, _, c in assigned[1:]:
                send_frame(c, self.key, K_UID, 0, uid, magic=MAGIC_RDV)
            self._conns = [c for _, _, c in assigned]
        except Exception as e:  # surfaced through .error
            self.error = repr(e)
        finally:
            for c in self._conns:
                try:
                    c.close()
                except OSError:
                    pass
            if self._sock is not None:
                self._sock.close()
            self._done.set()


def rendezvous(host: str, port: int, key: bytes, rank: int = -1, info: Optional[dict] = None,
               uid_fn: Optional[Callable[[], bytes]] = None,
               timeout: float = IDLE_TIMEOUT_S) -> RendezvousResult:
    """Join a rendezvous; returns this rank's (rank, world, uid, members)."""
    deadline = time.monotonic() + timeout
    while True:
        try:
            s = socket.create_connection((host, port), timeout=5.0)
            break
        except OSError:
            if time.monotonic() > deadline:
                raise
            time.sleep(0.05)
    s.settimeout(timeout)
    with s:
        hello = {"rank": rank, "host": socket.gethostname(), "info": info or {}}
        send_frame(s, key, K_HELLO, 0, json.dumps(hello).encode(), magic=MAGIC_RDV)
        kind, _, payload = recv_frame(s, key, magic=MAGIC_RDV, max_frame=MAX_RDV_FRAME)
        if kind == K_REJECT:
            raise ConnectionError(f"rendezvous rejected: {json.loads(payload)['reason']}")
        role = json.loads(payload.decode())
        if role["role"] == "generate":
            uid = (uid_fn or (lambda: os.urandom(128)))()
            send_frame(s, key, K_UID, 0, uid, magic=MAGIC_RDV)
        else:
            kind, _, uid = recv_frame(s, key, magic=MAGIC_RDV, max_frame=MAX_RDV_FRAME)
            if kind != K_UID:
                raise ConnectionError("expected UID")
    return RendezvousResult(role["rank"], role["world"], uid, role["members"])
