"""Coordinator-driven cluster runtime: the scheduler that decides when ranks
average, the ranks that follow its control messages, and survivor re-formation
when a rank leaves.

Reference roles: the cluster coordinator's event loop (flodl/src/distributed/
cluster_coordinator/event_loop.rs: ``tick``, ``should_average``),
``trigger_averaging`` (averaging.rs), progressive epoch dispatch from a chunk
pool (epoch_dispatch.rs, chunk_pool.rs), dead-rank detection (dead_ranks.rs),
the worker's control dispatch (ddp_run/worker/control.rs) and the NCCL
abort/rebuild retry of ``sync_now_nccl`` (ddp_run/worker/sync.rs:781-1031).

Processes: the coordinator runs as a thread of the launching process (or of
rank 0 for the cooperative tier); every rank is one process with one control
connection to it, carrying HMAC-signed frames of the native wire codec with
JSON bodies. Heartbeats ride the same connection from a background thread.

Control protocol (coordinator <-> rank):

    HELLO {rank}                       rank -> coord, once
    PLAN {wid, epoch, spans, batches}  coord -> rank: train these permutation
                                       spans, at most `batches` batches
    DONE {wid, batches, wall_ms, first_ms, samples, loss_sum, n_loss}
    SYNC {round, attempt}              coord -> rank: average now
    SYNCED {round, ok, sync_ms, div, err}
    SESSION {session, port, ranks}     coord -> survivors: rebuild the process
                                       group (rank = index in `ranks`) and the
                                       device communicator, then REBUILT
    EPOCH {epoch, callback_rank, save} coord -> rank: epoch finished
    EPOCH_ACK {epoch}
    HEARTBEAT {}                       rank -> coord
    BYE {}                             rank -> coord: leaving between windows
    DEAD {rank}                        coord -> ranks
    STOP {}                            coord -> ranks

Decisions (``Coordinator.tick``):

* A window is complete for a rank when it ran its ElChe batch count (Sync: one
  batch) or the epoch's pool has nothing left for it. ``should_average`` holds
  once every live rank's window is complete and at least one rank moved.
* ``trigger_averaging`` sends SYNC to every live rank; their SYNCED replies
  (sync time, divergence) feed ElChe's ``report_timing`` and the convergence
  guard, whose verdict commits, vetoes or discards ElChe's growth proposal.
* CpuAsync: a rank that finished its window while a slower one still trains
  gets up to ``max_overshoot`` more batches instead of idling.
* A rank whose heartbeat is older than ``heartbeat_timeout`` is dead; a rank
  that sends BYE leaves between windows. Its outstanding chunks go back to the
  pool, and survivors re-form (SESSION) before the next collective. A round
  that failed (a peer wait ran out, a gloo timeout) is retried on the
  re-formed session after each rank restored its pre-round parameters, up to
  ``MAX_REBUILD_ATTEMPTS`` times.
"""
from __future__ import annotations

import json
import queue
import socket
import threading
import time
from typing import Any, Callable, Dict, List, Optional, Tuple

from .cpu_reduce import recv_frame, send_frame

CTL_MAGIC = 0x464C4354  # "FLCT"
MAX_REBUILD_ATTEMPTS = 32

(K_HELLO, K_PLAN, K_DONE, K_SYNC, K_SYNCED, K_SESSION, K_REBUILT, K_EPOCH, K_EPOCH_ACK,
 K_HEARTBEAT, K_BYE, K_DEAD, K_STOP) = range(1, 14)

KIND_NAMES = {K_HELLO: "hello", K_PLAN: "plan", K_DONE: "done", K_SYNC: "sync",
              K_SYNCED: "synced", K_SESSION: "session", K_REBUILT: "rebuilt", K_EPOCH: "epoch",
              K_EPOCH_ACK: "epoch_ack", K_HEARTBEAT: "heartbeat", K_BYE: "bye", K_DEAD: "dead",
              K_STOP: "stop"}


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class ControlLink:
    """One signed-frame control connection (either side)."""

    def __init__(self, sock: socket.socket, key: bytes):
        self.sock, self.key = sock, key
        self.lock = threading.Lock()
        self.seq = 0

    def send(self, kind: int, body: Optional[dict] = None) -> None:
        self.seq += 1
        send_frame(self.sock, self.key, kind, self.seq, json.dumps(body or {}).encode(),
                   self.lock, magic=CTL_MAGIC)

    def recv(self) -> Tuple[int, dict]:
        kind, _seq, payload = recv_frame(self.sock, self.key, magic=CTL_MAGIC, max_frame=1 << 24)
        return kind, json.loads(payload.decode() or "{}")

    def close(self) -> None:
        try:
            self.sock.close()
        except OSError:
            pass


# ============================================================================ coordinator
class Coordinator:
    """The cluster scheduler. ``start()`` binds and runs the event loop on a
    thread; ``result()`` waits for the run to end and returns the record."""

    def __init__(self, world: int, key: bytes, dataset_len: int, cfg, seed: int = 0,
                 host: str = "127.0.0.1"):
        from .._ext import native
        from .config import ApplyPolicy
        from .convergence import GrowthGuard, LevelGuard, NoGuard  # noqa: F401
        from .meta import LrEventMeta

        self.world, self.key, self.cfg = world, key, cfg
        self.n = int(dataset_len)
        self.seed = seed
        self.bs = int(cfg.batch_size_)
        ec = cfg.elche_
        self.ec = ec
        self.policy, self.backend = ec.mode_.split()
        self.host = host
        self.srv = socket.socket()
        self.srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.srv.bind((host, 0))
        self.srv.listen(world + 8)
        self.port = self.srv.getsockname()[1]
        self.links: Dict[int, ControlLink] = {}
        self.inbox: "queue.Queue[Tuple[int, int, dict]]" = queue.Queue()
        self.alive = set(range(world))
        self.dead: List[int] = []
        self.last_seen: Dict[int, float] = {}
        self.hb_timeout = float(cfg.heartbeat_timeout_secs_)
        self.anchor_init = 1 if self.policy == ApplyPolicy.SYNC else int(ec.anchor_)
        self.elche = native().ElChe(world, self.anchor_init)
        if ec.overhead_target_:
            self.elche.set_overhead_target(ec.overhead_target_)
        if ec.max_anchor_:
            self.elche.set_max_anchor(ec.max_anchor_)
        if ec.min_anchor_:
            self.elche.set_min_anchor(ec.min_anchor_)
        if ec.max_batch_diff_:
            self.elche.set_max_batch_diff(ec.max_batch_diff_)
        if ec.partition_ratios_:
            self.elche.set_partition_ratios([float(x) for x in ec.partition_ratios_])
        self.elche.set_growth_applicable(self.policy != ApplyPolicy.SYNC)
        self.batches_per_epoch = max(1, -(-self.n // self.bs))
        self.elche.set_max_total(self.batches_per_epoch)
        if not ec.divergence_guard_:
            self.guard = NoGuard()
        else:
            self.guard = LevelGuard(ec.divergence_threshold_)
        self.meta = LrEventMeta() if ec.meta_controller_ else None
        self.record: Dict[str, Any] = {"batch_counts": [], "divergence": [], "syncs": 0,
                                       "verdicts": [], "anchors": [], "deaths": [],
                                       "sessions": 0, "retries": 0, "epochs": [],
                                       "windows_per_rank": [0] * world, "overshoot": 0}
        self.session = 0
        self.error: Optional[str] = None
        self._done = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.epoch = 0
        self.start_epoch = 0
        self.pool = None
        self.wid = 0
        self.round = 0
        self.cpu_ctl = None
        self.report_rank = 0

    # ---------------------------------------------------------------- plumbing
    def address(self) -> Tuple[str, int]:
        return self.host, self.port

    def start(self) -> "Coordinator":
        threading.Thread(target=self._accept, daemon=True).start()
        self._thread = threading.Thread(target=self._run_guarded, daemon=True)
        self._thread.start()
        return self

    def result(self, timeout: float = 3600.0) -> Dict[str, Any]:
        self._done.wait(timeout)
        if self.error:
            raise RuntimeError(f"coordinator: {self.error}")
        return self.record

    def _accept(self) -> None:
        while not self._done.is_set():
            try:
                self.srv.settimeout(0.5)
                c, _ = self.srv.accept()
            except socket.timeout:
                continue
            except OSError:
                return
            c.settimeout(None)
            link = ControlLink(c, self.key)
            try:
                kind, body = link.recv()
            except Exception:
                link.close()
                continue
            if kind != K_HELLO:
                link.close()
                continue
            rank = int(body["rank"])
            self.links[rank] = link
            self.last_seen[rank] = time.time()
            self.inbox.put((rank, K_HELLO, body))
            threading.Thread(target=self._reader, args=(rank, link), daemon=True).start()

    def _reader(self, rank: int, link: ControlLink) -> None:
        while True:
            try:
                kind, body = link.recv()
            except Exception:
                self.inbox.put((rank, -1, {}))  # connection lost
                return
            self.last_seen[rank] = time.time()
            if kind != K_HEARTBEAT:
                self.inbox.put((rank, kind, body))
            if kind == K_BYE:
                return

    def _send(self, rank: int, kind: int, body: Optional[dict] = None) -> None:
        link = self.links.get(rank)
        if link is None:
            return
        try:
            link.send(kind, body)
        except OSError:
            pass

    def _broadcast(self, kind: int, body: Optional[dict] = None) -> None:
        for r in sorted(self.alive):
            self._send(r, kind, body)

    def _next(self, want: Optional[set] = None, timeout: float = 0.1):
        """One inbox message (rank, kind, body), or None; runs the heartbeat
        watchdog while waiting."""
        try:
            return self.inbox.get(timeout=timeout)
        except queue.Empty:
            self._watchdog()
            return None

    def _watchdog(self) -> None:
        now = time.time()
        for r in list(self.alive):
            t = self.last_seen.get(r)
            if t is not None and now - t > self.hb_timeout:
                self._declare_dead(r, "heartbeat stale")

    def _declare_dead(self, r: int, why: str) -> None:
        if r not in self.alive:
            return
        self.alive.discard(r)
        self.dead.append(r)
        self.record["deaths"].append({"rank": r, "why": why, "epoch": self.epoch,
                                      "window": self.wid})
        if self.pool is not None:
            self.pool.forfeit(r)
        if self.cpu_ctl is not None:
            self.cpu_ctl._declare_dead(r)
        link = self.links.pop(r, None)
        if link is not None:
            link.close()
        self._broadcast(K_DEAD, {"rank": r})
        self._needs_session = True

    # ---------------------------------------------------------------- event loop
    def _run_guarded(self) -> None:
        try:
            self._run()
        except Exception as e:  # pragma: no cover - surfaced by result()
            import traceback
            self.error = f"{e!r}\n{traceback.format_exc()}"
            try:
                self._broadcast(K_STOP, {"error": repr(e)})
            except Exception:
                pass
        finally:
            self._done.set()
            try:
                self.srv.close()
            except OSError:
                pass

    def _wait_hello(self) -> None:
        got = set()
        deadline = time.time() + max(120.0, self.hb_timeout * 4)
        while got != set(range(self.world)):
            if time.time() > deadline:
                raise TimeoutError(f"ranks {sorted(set(range(self.world)) - got)} never connected")
            m = self._next()
            if m and m[1] == K_HELLO:
                got.add(m[0])

    def _run(self) -> None:
        from .config import AverageBackend
        self._needs_session = False
        if self.backend == AverageBackend.CPU and self.world > 1:
            # the CPU averaging backend's reduce controller lives beside the scheduler
            from .cpu_reduce import CpuReduceController
            self.cpu_ctl = CpuReduceController(self.world, self.key,
                                               heartbeat_timeout=self.hb_timeout)
        self._wait_hello()
        if self.cfg.resume_from_:
            self.start_epoch = int(self._resume_epoch())
        self._reform()  # the first session: process group, communicator, initial broadcast
        for epoch in range(self.start_epoch, int(self.cfg.num_epochs_)):
            if not self.alive:
                break
            self.epoch = epoch
            self._run_epoch(epoch)
        self.report_rank = min(self.alive) if self.alive else -1
        self._broadcast(K_STOP, {"report_rank": self.report_rank})
        if self.cpu_ctl is not None:
            self.cpu_ctl.close()

    def _resume_epoch(self) -> int:
        from .bundle import read_meta
        meta = read_meta(self.cfg.resume_from_)
        if meta.elche_state is not None and meta.world_size_at_save == self.world:
            st = meta.elche_state
            self.elche.restore_from_state({"anchor": st.anchor, "anchor_rank": st.anchor_rank,
                                           "smoothed_ms_per_batch": list(st.smoothed_ms_per_batch),
                                           "phase": st.phase,
                                           "calibration_count": st.calibration_count})
        return meta.epoch + 1

    def _spans(self) -> List[int]:
        from .coordinator import spans_from_throughput
        share = list(self.elche.recent_batch_share()) if self.elche.is_calibrated() else None
        if self.ec.partition_ratios_:
            share = [float(x) for x in self.ec.partition_ratios_]
        rates = [(share[r] if share else 1.0) if r in self.alive else 0.0
                 for r in range(self.world)]
        if not any(rates):
            rates = [1.0 if r in self.alive else 0.0 for r in range(self.world)]
        tot = sum(rates)
        out = [int(self.n * x / tot) for x in rates]
        last = max(r for r in range(self.world) if rates[r] > 0)
        out[last] += self.n - sum(out)
        return out

    def _plan_for(self, r: int, batches: int) -> Optional[dict]:
        """Take `batches` batches of samples for rank r from the pool."""
        want = batches * self.bs
        spans = []
        got = 0
        while got < want:
            ch = self.pool.take_chunk(want - got, r)
            if ch is None:
                break
            spans.append([int(ch[0]), int(ch[1])])
            got += int(ch[1])
        if not spans:
            return None
        return {"wid": self.wid, "epoch": self.epoch, "spans": spans,
                "batches": -(-got // self.bs), "samples": got}

    def _run_epoch(self, epoch: int) -> None:
        from .coordinator import ChunkPool
        from .config import ApplyPolicy

        self.pool = ChunkPool(epoch, self.n, self._spans())
        quiesced = set()
        while True:
            # ------------------------------------------------ dispatch one window
            if self._needs_session:
                self._reform()
            self.wid += 1
            counts = list(self.elche.batch_counts())
            if self.policy == ApplyPolicy.SYNC:
                counts = [1] * self.world
            ran: Dict[int, dict] = {}
            pending = set()
            for r in sorted(self.alive):
                plan = self._plan_for(r, counts[r])
                if plan is None:
                    quiesced.add(r)
                    continue
                self._send(r, K_PLAN, plan)
                pending.add(r)
            if not pending:
                break  # epoch exhausted
            overshoot_left = {r: int(self.ec.max_overshoot_) for r in pending}
            while pending & self.alive:
                m = self._next()
                if m is None:
                    continue
                r, kind, body = m
                if kind == -1 or kind == K_BYE:
                    self._declare_dead(r, "left" if kind == K_BYE else "connection lost")
                    pending.discard(r)
                    continue
                if kind != K_DONE or body.get("wid") != self.wid:
                    continue
                prev = ran.get(r)
                if prev is None:
                    ran[r] = dict(body)
                else:  # an overshoot extension of this window
                    for k in ("batches", "samples", "wall_ms", "loss_sum", "n_loss"):
                        prev[k] = prev.get(k, 0) + body.get(k, 0)
                self.pool.mark_completed(r, int(body.get("samples", 0)))
                self.record["windows_per_rank"][r] += 1
                # CpuAsync: a rank that finished early keeps training (bounded)
                if (self.policy == ApplyPolicy.ASYNC and overshoot_left.get(r, 0) > 0
                        and len(pending - {r}) > 0):
                    ext = self._plan_for(r, 1)
                    if ext is not None:
                        overshoot_left[r] -= 1
                        self.record["overshoot"] += 1
                        self._send(r, K_PLAN, ext)
                        continue
                pending.discard(r)
            if not self.alive:
                return
            if not any(int(b.get("batches", 0)) > 0 for r, b in ran.items() if r in self.alive):
                continue
            # ------------------------------------------------ average
            self._average(ran)
            if self.pool.is_epoch_done() and self.pool.remaining() == 0:
                break
        # ------------------------------------------------ epoch end
        self._epoch_end(epoch)

    def _reform(self) -> None:
        """Survivors rebuild their process group and device communicator."""
        self._needs_session = False
        self.session += 1
        self.record["sessions"] += 1
        ranks = sorted(self.alive)
        port = _free_port()
        body = {"session": self.session, "port": port, "ranks": ranks}
        if self.cpu_ctl is not None:
            body["cpu_port"] = self.cpu_ctl.port
        self._broadcast(K_SESSION, body)
        waiting = set(ranks)
        deadline = time.time() + max(120.0, 4 * self.hb_timeout)
        while waiting & self.alive:
            if time.time() > deadline:
                raise TimeoutError("survivors did not re-form")
            m = self._next()
            if m is None:
                continue
            r, kind, body = m
            if kind in (-1, K_BYE):
                self._declare_dead(r, "lost during re-formation")
                self._needs_session = True
            elif kind == K_REBUILT and body.get("session") == self.session:
                waiting.discard(r)
        if self._needs_session:
            self._reform()

    def _average(self, ran: Dict[int, dict]) -> None:
        self.round += 1
        attempt = 0
        while True:
            attempt += 1
            if self._needs_session:
                self._reform()
            self._broadcast(K_SYNC, {"round": self.round, "attempt": attempt})
            waiting = set(self.alive)
            replies: Dict[int, dict] = {}
            failed = False
            while waiting & self.alive:
                m = self._next()
                if m is None:
                    continue
                r, kind, body = m
                if kind in (-1, K_BYE):
                    self._declare_dead(r, "left" if kind == K_BYE else "connection lost")
                    failed = True
                    continue
                if kind == K_SYNCED and body.get("round") == self.round:
                    replies[r] = body
                    waiting.discard(r)
                    if not body.get("ok", True):
                        failed = True
            if not self.alive:
                return
            if not failed and not self._needs_session:
                break
            self.record["retries"] += 1
            if attempt >= MAX_REBUILD_ATTEMPTS:
                raise RuntimeError(f"averaging round {self.round} failed {attempt} times")
            self._needs_session = True
        self.record["syncs"] += 1
        sync_ms = max(float(b.get("sync_ms", 0.0)) for b in replies.values())
        div = max(float(b.get("div", 0.0)) for b in replies.values())
        self.record["divergence"].append(div)
        # ElChe: marginal per-batch wall (first batch = fill excluded)
        wall = [0.0] * self.world
        nb = [0] * self.world
        fill = [0.0] * self.world
        for r, b in ran.items():
            if r not in self.alive:
                continue
            n = int(b.get("batches", 0))
            w = float(b.get("wall_ms", 0.0))
            first = float(b.get("first_ms", 0.0))
            nb[r] = n
            wall[r] = w
            if n >= 2:
                marginal = (w - first) / (n - 1)
                fill[r] = max(0.0, first - marginal)
        self.elche.set_window_fill_ms(fill)
        self.elche.report_timing(wall, nb, sync_ms)
        verdict = self.guard.observe(div)
        from .convergence import Verdict
        if verdict == Verdict.STABLE:
            self.elche.apply_verdict("stable", 1.0, bool(self.ec.relax_up_))
        elif verdict == Verdict.SUPPRESS:
            self.elche.apply_verdict("suppress", 1.0, False)
        else:
            self.elche.apply_verdict("nudge", float(getattr(self.guard, "nudge_factor", 0.5)), False)
        if self.meta is not None:
            lrs = [float(b.get("lr", 0.0)) for b in replies.values()]
            f = self.meta.observe(lrs[0] if lrs else 0.0, int(self.elche.anchor()),
                                  {Verdict.STABLE: "stable", Verdict.SUPPRESS: "suppress_growth",
                                   Verdict.NUDGE: "shrink"}[verdict], self.elche.phase())
            if f is not None:
                self.elche.apply_verdict("nudge", float(f), False)
                self.record.setdefault("meta_nudges", []).append(float(f))
        self.record["verdicts"].append(verdict.value)
        self.record["anchors"].append(int(self.elche.anchor()))
        self.record["batch_counts"].append([nb[r] for r in range(self.world)])

    def _epoch_end(self, epoch: int) -> None:
        from .coordinator import CallbackRoles
        roles = getattr(self, "_roles", None)
        if roles is None:
            roles = self._roles = CallbackRoles(self.world)
        for r in self.dead:
            roles.rank_died(r)
        per = {r: self.elche.smoothed_ms(r) for r in self.alive}
        holder = roles.observe(per)
        save = bool(self.cfg.save_path_ and self.cfg.checkpoint_every_ and
                    (epoch + 1) % int(self.cfg.checkpoint_every_) == 0)
        st = dict(self.elche.to_state())
        body = {"epoch": epoch, "callback_rank": holder, "save": save,
                "elche_state": st, "syncs": self.record["syncs"],
                "coverage": [[int(a), int(b)] for a, b in self.pool.uncovered_ranges()]}
        self._broadcast(K_EPOCH, body)
        waiting = set(self.alive)
        while waiting & self.alive:
            m = self._next()
            if m is None:
                continue
            r, kind, b = m
            if kind in (-1, K_BYE):
                self._declare_dead(r, "left" if kind == K_BYE else "connection lost")
            elif kind == K_EPOCH_ACK and b.get("epoch") == epoch:
                waiting.discard(r)
        self.record["epochs"].append({"epoch": epoch, "callback_rank": holder,
                                      "alive": sorted(self.alive)})


# ============================================================================ rank side
class RankAgent:
    """The rank's end of the control connection plus its heartbeat thread."""

    def __init__(self, host: str, port: int, key: bytes, rank: int, heartbeat_s: float = 1.0):
        self.rank = rank
        sock = socket.create_connection((host, port), timeout=60)
        sock.settimeout(None)
        self.link = ControlLink(sock, key)
        self.link.send(K_HELLO, {"rank": rank})
        self._stop = threading.Event()
        self.hb_s = heartbeat_s
        self._hb = threading.Thread(target=self._heartbeat, daemon=True)
        self._hb.start()

    def _heartbeat(self) -> None:
        while not self._stop.wait(self.hb_s):
            try:
                self.link.send(K_HEARTBEAT, {})
            except OSError:
                return

    def pause_heartbeat(self) -> None:
        """Stop heart-beating (a test stand-in for a rank that hangs)."""
        self._stop.set()

    def send(self, kind: int, body: Optional[dict] = None) -> None:
        self.link.send(kind, body)

    def recv(self) -> Tuple[int, dict]:
        return self.link.recv()

    def close(self, bye: bool = False) -> None:
        self._stop.set()
        if bye:
            try:
                self.link.send(K_BYE, {})
            except OSError:
                pass
        self.link.close()
