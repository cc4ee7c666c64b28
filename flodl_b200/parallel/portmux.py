"""One accepting port for every controller channel, plus the run-status board.

Reference: flodl/src/distributed/port_mux.rs (channel-select dispatch by the
first four bytes of a connection), status.rs (``state.json`` over plain HTTP
on the same port, ``POST /start`` operator switch) and bind_diag.rs (who holds
a busy port).

Dialers of the signed wire protocol open with the frame magic (the first
field of every frame header, little-endian u32). The dispatcher peeks those
four bytes without consuming them and hands the connection to the subsystem
registered for that magic, which then reads a byte-identical stream - a
directly bound listener and a muxed one are interchangeable. ``GET `` and
``POST`` route to the status responder. A connection that sends nothing
within the peek deadline, or an unknown magic, is closed; the dispatcher
moves on.
"""
from __future__ import annotations

import errno
import json
import os
import socket
import struct
import threading
import time
from typing import Callable, Dict, Optional
from urllib.parse import parse_qs, urlparse

HTTP_GET = b"GET "
HTTP_POST = b"POST"


def magic_bytes(magic: int) -> bytes:
    return struct.pack("<I", magic)


class PortMux:
    def __init__(self, host: str = "127.0.0.1", port: int = 0, peek_timeout: float = 5.0):
        self.sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self.sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        try:
            self.sock.bind((host, port))
        except OSError as e:
            if e.errno == errno.EADDRINUSE:
                raise OSError(e.errno, f"port {port} is busy: {describe_port_holder(port)}") from e
            raise
        self.sock.listen(256)
        self.host, self.port = self.sock.getsockname()
        self.peek_timeout = peek_timeout
        self.routes: Dict[bytes, Callable[[socket.socket], None]] = {}
        self.dropped = 0
        self._stop = threading.Event()
        threading.Thread(target=self._dispatch, daemon=True).start()

    def route(self, prefix: bytes, handler: Callable[[socket.socket], None]) -> None:
        if len(prefix) != 4:
            raise ValueError("a channel-select prefix is four bytes")
        self.routes[prefix] = handler

    def route_magic(self, magic: int, handler: Callable[[socket.socket], None]) -> None:
        self.route(magic_bytes(magic), handler)

    def serve_status(self, board: "StatusBoard") -> None:
        h = lambda c: threading.Thread(target=_serve_http, args=(c, board), daemon=True).start()
        self.route(HTTP_GET, h)
        self.route(HTTP_POST, h)

    def _peek4(self, c: socket.socket) -> Optional[bytes]:
        c.settimeout(self.peek_timeout)
        deadline = time.monotonic() + self.peek_timeout
        while time.monotonic() < deadline:
            try:
                b = c.recv(4, socket.MSG_PEEK)
            except (socket.timeout, OSError):
                return None
            if not b:
                return None
            if len(b) == 4:
                return b
            time.sleep(0.002)
        return None

    def _dispatch(self) -> None:
        while not self._stop.is_set():
            try:
                c, _ = self.sock.accept()
            except OSError:
                return
            head = self._peek4(c)
            handler = self.routes.get(head) if head else None
            if handler is None:
                self.dropped += 1
                c.close()
                continue
            c.settimeout(None)
            try:
                handler(c)
            except Exception:
                self.dropped += 1
                c.close()

    def close(self) -> None:
        self._stop.set()
        try:
            self.sock.close()
        except OSError:
            pass


class StatusBoard:
    """Latest membership snapshot, served as ``state.json``; holds the
    operator start switch for Manual/Hybrid starts."""

    def __init__(self):
        self._lock = threading.Lock()
        self._state: Optional[dict] = None
        self._start_mode = None
        self._token = ""
        self._start = threading.Event()
        self.dashboard_port: Optional[int] = None
        self.quorum_ok: Callable[[], bool] = lambda: True

    def publish(self, snapshot: dict) -> None:
        with self._lock:
            self._state = dict(snapshot, published_at=time.time())

    def set_dashboard_port(self, port: int) -> None:
        with self._lock:
            self.dashboard_port = port

    def state_json(self) -> Optional[str]:
        with self._lock:
            if self._state is None:
                return None
            st = dict(self._state)
            if self.dashboard_port is not None:
                st["dashboard_port"] = self.dashboard_port
            st["start_requested"] = self._start.is_set()
            return json.dumps(st)

    def configure_start(self, mode, token_hex: str) -> None:
        self._start_mode, self._token = mode, token_hex

    def start_requested(self) -> bool:
        return self._start.is_set()

    def request_start(self, peer_host: str, token: str) -> tuple:
        """(HTTP status, message). Loopback peers are trusted; others need the token."""
        if self._start_mode is None or getattr(self._start_mode, "value", "auto") == "auto":
            return 409, "run does not use a manual start"
        loopback = peer_host.startswith("127.") or peer_host == "::1"
        if not loopback and (not self._token or token != self._token):
            return 403, "start needs the session token"
        if not self.quorum_ok():
            return 409, "quorum not reached"
        self._start.set()
        return 200, "start armed"


def _serve_http(c: socket.socket, board: StatusBoard) -> None:
    try:
        c.settimeout(5.0)
        peer = c.getpeername()[0]
        data = b""
        while b"\r\n\r\n" not in data and len(data) < 16384:
            chunk = c.recv(4096)
            if not chunk:
                break
            data += chunk
        line = data.split(b"\r\n", 1)[0].decode("latin-1")
        parts = line.split(" ")
        method, target = (parts[0], parts[1]) if len(parts) >= 2 else ("", "/")
        url = urlparse(target)
        if method == "GET" and url.path in ("/", "/state.json"):
            body = board.state_json()
            code, ctype = (200, "application/json") if body else (503, "text/plain")
            body = body or "no snapshot published yet"
        elif method == "GET" and url.path == "/healthz":
            code, ctype, body = 200, "text/plain", "ok"
        elif method == "POST" and url.path == "/start":
            token = parse_qs(url.query).get("token", [""])[0]
            code, body = board.request_start(peer, token)
            ctype = "text/plain"
        else:
            code, ctype, body = 404, "text/plain", "not found"
        reason = {200: "OK", 403: "Forbidden", 404: "Not Found", 409: "Conflict",
                  503: "Service Unavailable"}[code]
        raw = body.encode()
        c.sendall(f"HTTP/1.1 {code} {reason}\r\nContent-Type: {ctype}\r\n"
                  f"Content-Length: {len(raw)}\r\nConnection: close\r\n\r\n".encode() + raw)
    except OSError:
        pass
    finally:
        c.close()


# ----------------------------------------------------------------- bind diagnosis
def _listening_inodes(port: int) -> Dict[str, str]:
    """socket inode -> local address for TCP sockets listening on ``port``."""
    out = {}
    for fn in ("/proc/net/tcp", "/proc/net/tcp6"):
        try:
            with open(fn) as f:
                next(f)
                for line in f:
                    cols = line.split()
                    local, state, inode = cols[1], cols[3], cols[9]
                    if state == "0A" and int(local.rsplit(":", 1)[1], 16) == port:
                        out[inode] = local
        except (OSError, StopIteration):
            continue
    return out


def port_holders(port: int) -> list:
    """[(pid, command line)] of processes holding a listening socket on ``port``
    (the ones this user may inspect)."""
    inodes = _listening_inodes(port)
    if not inodes:
        return []
    found = []
    for pid in filter(str.isdigit, os.listdir("/proc")):
        fd_dir = f"/proc/{pid}/fd"
        try:
            fds = os.listdir(fd_dir)
        except OSError:
            continue
        for fd in fds:
            try:
                link = os.readlink(f"{fd_dir}/{fd}")
            except OSError:
                continue
            if link.startswith("socket:[") and link[8:-1] in inodes:
                try:
                    with open(f"/proc/{pid}/cmdline", "rb") as f:
                        cmd = f.read().replace(b"\0", b" ").decode(errors="replace").strip()
                except OSError:
                    cmd = "?"
                found.append((int(pid), cmd))
                break
    return found


def describe_port_holder(port: int) -> str:
    h = port_holders(port)
    if not h:
        return "held by a process this user cannot inspect (or in TIME_WAIT)"
    return "; ".join(f"pid {p}: {cmd[:120]}" for p, cmd in h)
