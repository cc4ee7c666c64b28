"""Process launcher: roles, local fan-out, supervision and elastic shrink.

Reference: flodl/src/distributed/launcher/mod.rs:116-240 (``Role`` from the
``FLODL_INTERNAL_*`` environment envelope; fan-out by local fork+exec or SSH;
supervision; elastic shrink) and spawn.rs.

One process per device. The launcher runs a :class:`RendezvousServer`, starts
one child per device with the role envelope in its environment, and watches
them. A child calls :func:`init_rank`, which joins the rendezvous - rank 0
generates the torch.distributed address, the others receive it - and
initialises the process group (NCCL for CUDA devices, gloo for CPU ranks).

Failure policy: ``abort`` stops the job at the first failed rank; ``shrink``
records a death record for it, stops the survivors and relaunches the job
with one rank less (membership only shrinks), up to ``max_restarts`` times -
the job is expected to resume from its last checkpoint bundle.

Remote hosts: :meth:`LocalLauncher.remote_command` builds the ``ssh`` command
line that starts the same role envelope on another host (fan-out over SSH);
with dial-in membership the host runs ``python -m flodl_b200.parallel.agent``
instead (:mod:`flodl_b200.parallel.agent`), which joins the controller's window
and spawns the host's ranks itself.
"""
from __future__ import annotations

import enum
import json
import os
import secrets
import shlex
import socket
import subprocess
import sys
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

from .rendezvous import RendezvousServer, rendezvous

ENV_ROLE = "FLODL_INTERNAL_ROLE"
ENV_RDV = "FLODL_INTERNAL_RDV"          # host:port of the rendezvous
ENV_KEY = "FLODL_INTERNAL_KEY"          # hex job key (signs every wire frame)
ENV_DEVICE = "FLODL_INTERNAL_DEVICE"    # device of this rank ("cuda:3", "cpu")
ENV_WORLD = "FLODL_INTERNAL_WORLD"
ENV_ATTEMPT = "FLODL_INTERNAL_ATTEMPT"


class Role(enum.Enum):
    SingleDevice = "single"
    Rank = "rank"
    Launcher = "launcher"
    Relay = "relay"
    Agent = "agent"


def role_from_env(env=None) -> Role:
    env = os.environ if env is None else env
    v = env.get(ENV_ROLE)
    if v:
        return Role(v)
    if int(env.get("WORLD_SIZE", "1")) > 1:
        return Role.Rank
    return Role.SingleDevice


@dataclass
class RankInfo:
    rank: int
    world: int
    device: str
    members: List[dict] = field(default_factory=list)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def init_rank(backend: Optional[str] = None, timeout_s: float = 120.0) -> RankInfo:
    """In a launched child: rendezvous, then torch.distributed init."""
    import datetime

    import torch
    import torch.distributed as dist

    host, port = os.environ[ENV_RDV].rsplit(":", 1)
    key = bytes.fromhex(os.environ[ENV_KEY])
    device = os.environ.get(ENV_DEVICE, "cpu")
    want = int(os.environ.get("LOCAL_RANK", "-1"))

    def uid() -> bytes:
        return json.dumps({"master_addr": "127.0.0.1", "master_port": _free_port()}).encode()

    res = rendezvous(host, int(port), key, rank=want, info={"device": device}, uid_fn=uid,
                     timeout=timeout_s)
    addr = json.loads(res.uid.decode())
    os.environ.update(MASTER_ADDR=addr["master_addr"], MASTER_PORT=str(addr["master_port"]),
                      RANK=str(res.rank), WORLD_SIZE=str(res.world))
    if backend is None:
        backend = "nccl" if device.startswith("cuda") else "gloo"
    kw = {}
    if backend == "nccl":
        dev = torch.device(device)
        torch.cuda.set_device(dev)
        kw["device_id"] = dev
    dist.init_process_group(backend, rank=res.rank, world_size=res.world,
                            timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return RankInfo(res.rank, res.world, device, res.members)


@dataclass
class LaunchResult:
    ok: bool
    world: int
    attempts: int
    exit_codes: List[int]
    deaths: List[dict]


class LocalLauncher:
    """Fan a command out to one child per device on this host."""

    def __init__(self, command: Sequence[str], devices: Sequence[str], policy: str = "abort",
                 max_restarts: int = 1, env: Optional[Dict[str, str]] = None,
                 timeout_s: float = 3600.0, death_log: Optional[str] = None,
                 max_failure=None):
        """``max_failure``: a :class:`~flodl_b200.parallel.coordinator.MaxFailureThreshold`
        over the initial world; once breached, ``shrink`` stops relaunching."""
        if policy not in ("abort", "shrink"):
            raise ValueError("policy must be 'abort' or 'shrink'")
        self.command = list(command)
        self.devices = list(devices)
        self.policy, self.max_restarts = policy, max_restarts
        self.env = dict(env or {})
        self.timeout_s = timeout_s
        self.death_log = death_log
        self.max_failure = max_failure
        self.key = secrets.token_bytes(32)

    def _spawn(self, devices: List[str], rdv: RendezvousServer, attempt: int):
        procs = []
        for i, dev in enumerate(devices):
            env = dict(os.environ)
            env.update(self.env)
            env.update({ENV_ROLE: Role.Rank.value, ENV_RDV: f"{rdv.host}:{rdv.port}",
                        ENV_KEY: self.key.hex(), ENV_DEVICE: dev, ENV_WORLD: str(len(devices)),
                        ENV_ATTEMPT: str(attempt), "LOCAL_RANK": str(i)})
            procs.append(subprocess.Popen(self.command, env=env))
        return procs

    def run(self) -> LaunchResult:
        devices = list(self.devices)
        deaths: List[dict] = []
        attempt = 0
        while True:
            rdv = RendezvousServer(len(devices), self.key).start()
            procs = self._spawn(devices, rdv, attempt)
            t0 = time.monotonic()
            failed = None
            while True:
                codes = [p.poll() for p in procs]
                bad = [(i, c) for i, c in enumerate(codes) if c not in (None, 0)]
                if bad:
                    failed = bad[0]
                    break
                if all(c == 0 for c in codes):
                    break
                if time.monotonic() - t0 > self.timeout_s:
                    failed = (-1, -9)
                    break
                time.sleep(0.05)
            if failed is None:
                return LaunchResult(True, len(devices), attempt + 1, [p.returncode for p in procs],
                                    deaths)
            # stop the survivors of this attempt
            for p in procs:
                if p.poll() is None:
                    p.terminate()
            for p in procs:
                try:
                    p.wait(timeout=10)
                except subprocess.TimeoutExpired:
                    p.kill()
            idx, code = failed
            rec = {"attempt": attempt, "local_rank": idx, "exit_code": code,
                   "device": devices[idx] if idx >= 0 else None,
                   "reason": "timeout" if idx < 0 else "rank exited with an error",
                   "world": len(devices), "at": time.time()}
            deaths.append(rec)
            if self.death_log:
                with open(self.death_log, "a") as f:
                    f.write(json.dumps(rec) + "\n")
            breached = (self.max_failure is not None and
                        self.max_failure.breached(len(deaths), len(self.devices)))
            if (self.policy == "abort" or attempt >= self.max_restarts or idx < 0
                    or len(devices) <= 1 or breached):
                return LaunchResult(False, len(devices), attempt + 1,
                                    [p.returncode for p in procs], deaths)
            devices.pop(idx)  # elastic shrink: relaunch without the failed device
            attempt += 1

    @staticmethod
    def remote_command(host: str, command: Sequence[str], env: Dict[str, str]) -> List[str]:
        """ssh command line that runs ``command`` on ``host`` with the role envelope."""
        exports = " ".join(f"{k}={shlex.quote(v)}" for k, v in env.items())
        return ["ssh", host, f"env {exports} " + " ".join(shlex.quote(c) for c in command)]


def main():
    """``python -m flodl_b200.parallel.launcher --devices cpu,cpu -- python train.py``"""
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--devices", required=True)
    ap.add_argument("--policy", default="abort", choices=["abort", "shrink"])
    ap.add_argument("--max-restarts", type=int, default=1)
    ap.add_argument("command", nargs=argparse.REMAINDER)
    a = ap.parse_args()
    cmd = a.command[1:] if a.command and a.command[0] == "--" else a.command
    r = LocalLauncher(cmd, a.devices.split(","), a.policy, a.max_restarts).run()
    print(json.dumps(r.__dict__), flush=True)
    sys.exit(0 if r.ok else 1)


if __name__ == "__main__":
    main()
