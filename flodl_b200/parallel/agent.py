"""Dial-in membership: per-host agents join a controller's window, receive
their host envelope once the world forms, then run and supervise the ranks.

Reference: flodl/src/distributed/launcher/agent.rs (the worker-side half of
dial-in membership) and membership.rs (the controller's join window).

Join channel (signed frames, channel magic ``FLJN``, served directly or
through :class:`~flodl_b200.parallel.portmux.PortMux`):

    HELLO   agent -> controller  {"host", "devices", "info"}
    ASSIGN  controller -> agent  {"cluster": <per-host envelope>, "command", "env"}
    EXITED  agent -> controller  {"local": i, "rank": r, "code": c}
    ABORT   controller -> agent  {"reason"}
    DONE    agent -> controller  {}  (every local rank exited 0)

The controller (:class:`JoinServer`) admits agents into a
:class:`~flodl_b200.parallel.membership.JoinWindow`; when it forms, ranks are
numbered in join order (a host's devices take consecutive ranks) and each
agent receives the slim envelope for its host - the same
``FLODL_INTERNAL_CLUSTER_JSON`` a launcher would ship. A rank that exits
non-zero is reported with its rank (per-rank granularity for elastic
membership); the controller's failure policy answers ``abort`` (tear every
host down) or ``shrink`` (record it; the survivors continue). The agent
touches no CUDA: device counts come from :func:`flodl_b200.utils.hw.detect_gpus`.
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
import threading
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

from .cluster import ENV_CLUSTER_JSON, ENV_HOST_OVERRIDE, ENV_LOCAL_RANK, ClusterBuilder
from .cpu_reduce import recv_frame, send_frame
from .membership import ClusterPhase, JoinWindow, StartMode

MAGIC_JOIN = 0x464C4A4E  # "FLJN"
K_HELLO, K_ASSIGN, K_EXITED, K_ABORT, K_DONE = 1, 2, 3, 4, 5


def _send(sock, key, kind, obj, lock=None):
    send_frame(sock, key, kind, 0, json.dumps(obj).encode(), lock, magic=MAGIC_JOIN)


def _recv(sock, key):
    kind, _, payload = recv_frame(sock, key, magic=MAGIC_JOIN, max_frame=1 << 20)
    return kind, json.loads(payload.decode() or "{}")


@dataclass
class _Agent:
    host: str
    devices: int
    sock: socket.socket
    lock: threading.Lock = field(default_factory=threading.Lock)
    ranks: List[int] = field(default_factory=list)
    done: bool = False


class JoinServer:
    def __init__(self, key: bytes, expected_hosts: int, command: Sequence[str],
                 mode: StartMode = StartMode.Auto, min_hosts: int = 1, window_s: float = 120.0,
                 policy: str = "abort", env: Optional[Dict[str, str]] = None,
                 controller_host: str = "127.0.0.1", controller_port: int = 0,
                 host: str = "127.0.0.1", port: Optional[int] = 0):
        if policy not in ("abort", "shrink"):
            raise ValueError("policy must be 'abort' or 'shrink'")
        self.key, self.command, self.policy = key, list(command), policy
        self.env = dict(env or {})
        self.ctl = (controller_host, controller_port)
        self.window = JoinWindow(expected_hosts, mode, min_hosts, window_s)
        self.agents: Dict[str, _Agent] = {}
        self.exits: List[dict] = []
        self.aborted: Optional[str] = None
        self._lock = threading.Lock()
        self._all_done = threading.Event()
        self.srv = None
        self.port = None
        if port is not None:
            self.srv = socket.socket()
            self.srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            self.srv.bind((host, port))
            self.srv.listen(64)
            self.port = self.srv.getsockname()[1]
            threading.Thread(target=self._accept, daemon=True).start()
        threading.Thread(target=self._formation, daemon=True).start()

    def _accept(self):
        while True:
            try:
                c, _ = self.srv.accept()
            except OSError:
                return
            self.adopt(c)

    def adopt(self, c: socket.socket) -> None:
        threading.Thread(target=self._serve, args=(c,), daemon=True).start()

    def _serve(self, c: socket.socket):
        agent = None
        try:
            kind, hello = _recv(c, self.key)
            if kind != K_HELLO:
                raise ConnectionError("expected HELLO")
            name = hello["host"]
            if not self.window.join(name, name, int(hello.get("devices", 1))):
                _send(c, self.key, K_ABORT, {"reason": self.window.refused[-1][1]})
                c.close()
                return
            agent = _Agent(name, int(hello.get("devices", 1)), c)
            with self._lock:
                self.agents[name] = agent
            while True:
                kind, msg = _recv(c, self.key)
                if kind == K_EXITED:
                    self._rank_exited(agent, msg)
                elif kind == K_DONE:
                    agent.done = True
                    self._check_done()
                    return
        except (ConnectionError, OSError, ValueError):
            if agent is not None and not agent.done:
                self._rank_exited(agent, {"rank": None, "code": None, "reason": "agent connection lost"})
        finally:
            if agent is None:
                c.close()

    def _formation(self):
        while not self.window.wait_formed(0.1):
            if self.window.poll() is ClusterPhase.Failed:
                self.aborted = "join window expired below quorum"
                self._broadcast_abort(self.aborted)
                self._all_done.set()
                return
        members = sorted((m for m in self.window.members.values() if m.rank >= 0),
                         key=lambda m: m.rank)
        b = ClusterBuilder().controller(self.ctl[0]).port(self.ctl[1]).done()
        for m in members:
            b = b.host(m.name).ranks(range(m.rank, m.rank + m.devices)).all_devices().done()
        full = b.build().with_session_salt()
        self.cluster = full
        for m in members:
            a = self.agents[m.name]
            a.ranks = list(range(m.rank, m.rank + m.devices))
            _send(a.sock, self.key, K_ASSIGN,
                  {"cluster": full.envelope_for(m.name).to_json(), "command": self.command,
                   "env": self.env}, a.lock)

    def _rank_exited(self, agent: _Agent, msg: dict):
        rec = dict(msg, host=agent.host, at=time.time())
        with self._lock:
            self.exits.append(rec)
        if msg.get("code") == 0:
            return
        self.window.remove(agent.host, f"rank {msg.get('rank')} exited {msg.get('code')}")
        if self.policy == "abort" and self.aborted is None:
            self.aborted = f"rank {msg.get('rank')} on {agent.host} failed ({msg.get('code')})"
            self._broadcast_abort(self.aborted)
            self._all_done.set()

    def _broadcast_abort(self, reason: str):
        for a in list(self.agents.values()):
            try:
                _send(a.sock, self.key, K_ABORT, {"reason": reason}, a.lock)
            except OSError:
                pass

    def _check_done(self):
        with self._lock:
            alive = [a for a in self.agents.values() if a.host in self.window.members
                     and self.window.members[a.host].alive]
            if alive and all(a.done for a in alive):
                self._all_done.set()

    def wait(self, timeout: Optional[float] = None) -> bool:
        """True when every surviving host finished cleanly."""
        self._all_done.wait(timeout)
        return self._all_done.is_set() and self.aborted is None

    def close(self):
        if self.srv is not None:
            self.srv.close()


def run_agent(controller: str, key: bytes, devices: Optional[int] = None, host: Optional[str] = None,
              info: Optional[dict] = None, timeout_s: float = 3600.0, log=print) -> int:
    """The per-host process: dial in, wait for the assignment, run and
    supervise the local ranks. Returns 0 when every local rank exited 0."""
    ch, cp = controller.rsplit(":", 1)
    host = host or os.environ.get(ENV_HOST_OVERRIDE) or socket.gethostname()
    if devices is None:
        from ..utils.hw import detect_gpus
        devices = max(1, len(detect_gpus()))
    sock = socket.create_connection((ch, int(cp)), timeout=30)
    sock.settimeout(None)
    lock = threading.Lock()
    _send(sock, key, K_HELLO, {"host": host, "devices": devices, "info": info or {}}, lock)
    kind, msg = _recv(sock, key)
    if kind == K_ABORT:
        log(f"[agent {host}] refused: {msg.get('reason')}")
        return 2
    if kind != K_ASSIGN:
        raise ConnectionError("expected ASSIGN")
    envelope = msg["cluster"]
    ranks = envelope["worker"]["ranks"]
    procs = []
    for i, r in enumerate(ranks):
        env = dict(os.environ)
        env.update({k: str(v) for k, v in (msg.get("env") or {}).items()})
        env.update({ENV_CLUSTER_JSON: json.dumps(envelope), ENV_LOCAL_RANK: str(i),
                    ENV_HOST_OVERRIDE: host, "RANK": str(r),
                    "WORLD_SIZE": str(envelope["world_size"])})
        procs.append(subprocess.Popen(msg["command"], env=env))
    aborted = threading.Event()

    def listen():
        try:
            k, m = _recv(sock, key)
            if k == K_ABORT:
                log(f"[agent {host}] abort: {m.get('reason')}")
                aborted.set()
        except (ConnectionError, OSError, ValueError):
            aborted.set()

    threading.Thread(target=listen, daemon=True).start()
    reported = set()
    t0 = time.monotonic()
    rc = 0
    while len(reported) < len(procs):
        for i, p in enumerate(procs):
            if i in reported:
                continue
            code = p.poll()
            if code is not None:
                reported.add(i)
                rc = rc or code
                try:
                    _send(sock, key, K_EXITED, {"local": i, "rank": ranks[i], "code": code}, lock)
                except OSError:
                    pass
        if aborted.is_set() or time.monotonic() - t0 > timeout_s:
            for p in procs:
                if p.poll() is None:
                    p.terminate()
            for p in procs:
                try:
                    p.wait(10)
                except subprocess.TimeoutExpired:
                    p.kill()
            return 3
        time.sleep(0.05)
    if rc == 0:
        try:
            _send(sock, key, K_DONE, {}, lock)
        except OSError:
            pass
    sock.close()
    return rc


def main():
    import argparse
    ap = argparse.ArgumentParser(description="per-host agent: join a controller and run its ranks")
    ap.add_argument("--controller", required=True, help="host:port of the controller (join channel)")
    ap.add_argument("--key-hex", default=os.environ.get("FLODL_INTERNAL_KEY", ""))
    ap.add_argument("--devices", type=int, default=None)
    a = ap.parse_args()
    sys.exit(run_agent(a.controller, bytes.fromhex(a.key_hex), a.devices))


if __name__ == "__main__":
    main()
