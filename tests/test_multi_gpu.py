"""Peer-memory collectives and fused DDP on 2, 4 and 8 GPUs of one node.

Each test spawns one process per GPU (NCCL bootstrap on 127.0.0.1, NVLS off
so no rank ever binds memory to a multicast object) and is skipped, with the
reason, when fewer GPUs are visible. Every result is checked against NCCL or
against a single-GPU run of the same model on the full batch.

Covered: two-shot and one-shot all-reduce at sizes that are not multiples of
world x 4, broadcast from a non-zero root, the weighted average with a
gamma-mass, an idle rank, an f32 buffer part averaged over the ranks that
moved, the divergence partials, and the all-idle no-op; fused DDP with AdamW
and SGD over at least three buckets that mix the one-shot and two-shot forms,
the bf16 shadow after the all-gather, global-norm clipping, and a
CUDA-graph-captured step against the eager one.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLDS = [2, 4, 8]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _need_gpus(n=2):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs (have {torch.cuda.device_count()})")


def _collect(q, procs, world, timeout=300.0):
    """Results from every worker; fails fast if a worker died without one."""
    import queue
    import time

    out = []
    deadline = time.monotonic() + timeout
    while len(out) < world:
        try:
            out.append(q.get(timeout=2.0))
            continue
        except queue.Empty:
            pass
        dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
        if dead:
            raise AssertionError(f"worker exited with code(s) {dead} before reporting")
        if time.monotonic() > deadline:
            raise AssertionError("workers did not report in time")
    return out


def _spawn(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(_collect(q, procs, world), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
    return res


def _init(rank, world, port):
    import datetime
    from flodl_b200.utils.crash import install_crash_handler

    install_crash_handler()

    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))


# ----------------------------------------------------------------------------- collectives
def _collectives_worker(rank, world, port, q):
    import torch.distributed as dist

    from flodl_b200.parallel.convergence import realized_mass
    from flodl_b200.parallel.peer import PeerComm

    checks = {}
    try:
        _init(rank, world, port)
        dev = torch.device("cuda", rank)
        nmax = (1 << 20) + 36
        comm = PeerComm(nmax + 64, dev, timeout_s=5.0)
        slot = 0
        for n in (1000, 4096 + 12, nmax):
            for oneshot in (False, True):
                g = torch.Generator(device="cuda").manual_seed(1000 * rank + n)
                x = torch.randn(n, device="cuda", generator=g)
                comm.grad[:n].copy_(x)
                ref = x.clone()
                dist.all_reduce(ref)
                comm.all_reduce_(n, average=False, slot=slot, oneshot=oneshot)
                slot += 1
                torch.cuda.synchronize()
                comm.check()
                checks[f"allreduce n={n} oneshot={oneshot}"] = bool(
                    torch.allclose(comm.grad[:n], ref, atol=1e-4, rtol=1e-5))
        # broadcast from the last rank; the shadow follows the pulled weights
        n = nmax
        comm.data[:n].fill_(float(rank + 1))
        comm.broadcast_(n, root=world - 1, slot=slot)
        slot += 1
        torch.cuda.synchronize()
        checks["broadcast"] = bool((comm.data[:n] == float(world)).all())
        checks["broadcast shadow"] = bool((comm.shadow[:n].float() == float(world)).all())
        # weighted average: gamma 0.5 mass, the last rank idle, a buffer tail
        gamma = 0.5
        nparam, nbuf = 100_000, 1000  # nparam is a multiple of 4
        n = nparam + nbuf
        g = torch.Generator(device="cuda").manual_seed(77 + rank)
        mine = torch.randn(n, device="cuda", generator=g)
        comm.data[:n].copy_(mine)
        batches = [0 if r == world - 1 else r + 1 for r in range(world)]
        masses = [realized_mass(b, gamma) for b in batches]
        allx = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allx, mine)
        X = torch.stack(allx).double()
        w = torch.tensor(masses, dtype=torch.float64, device="cuda")
        movers = torch.tensor([1.0 if b > 0 else 0.0 for b in batches], dtype=torch.float64,
                              device="cuda")
        expect = torch.empty(n, dtype=torch.float64, device="cuda")
        expect[:nparam] = (w[:, None] * X[:, :nparam]).sum(0) / w.sum()
        expect[nparam:] = (movers[:, None] * X[:, nparam:]).sum(0) / movers.sum()
        div = torch.zeros(2, device="cuda")
        comm.weighted_average_(n, masses[rank], slot=slot, div=div, buf_start=nparam)
        slot += 1
        torch.cuda.synchronize()
        comm.check()
        checks["weighted average"] = bool(torch.allclose(comm.data[:n].double(), expect,
                                                         atol=1e-5, rtol=1e-5))
        d2 = float(((X[rank, :nparam] - expect[:nparam]) ** 2).sum())
        p2 = float((expect[:nparam] ** 2).sum())
        checks["divergence partials"] = (abs(div[0].item() - d2) <= 1e-3 * max(d2, 1e-6)
                                         and abs(div[1].item() - p2) <= 1e-3 * p2)
        checks["weighted average shadow"] = bool(torch.equal(comm.shadow[:n],
                                                             comm.data[:n].bfloat16()))
        # nobody moved: nothing changes
        before = comm.data[:n].clone()
        comm.weighted_average_(n, 0.0, slot=slot, buf_start=nparam)
        torch.cuda.synchronize()
        comm.check()
        checks["all idle is a no-op"] = bool(torch.equal(before, comm.data[:n]))
        comm.close()
        q.put((rank, checks, None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, checks, traceback.format_exc()))


@pytest.mark.parametrize("world", WORLDS)
def test_peer_collectives(world):
    _need_gpus(world)
    for rank, checks, err in _spawn(_collectives_worker, world):
        assert err is None, err
        bad = [k for k, v in checks.items() if not v]
        assert not bad, f"rank {rank}: failed {bad}"


# ----------------------------------------------------------------------------- fused DDP
def _lm(dev):
    from flodl_b200.models import TransformerLM

    torch.manual_seed(0)
    return TransformerLM(vocab_size=256, d_model=256, n_layers=2, n_heads=4, d_ff=1024,
                         max_seq=128, device=dev)


def _batch(world, dev):
    g = torch.Generator(device="cuda").manual_seed(100)
    return torch.randint(0, 256, (4 * world, 128), device=dev, generator=g)


def _make_opt(kind, params):
    from flodl_b200.optim import SGD, AdamW

    if kind == "sgd":
        return SGD(params, lr=0.05, momentum=0.9, weight_decay=1e-4)
    if kind == "adamw2":
        # two parameter groups with their own lr / weight decay (matrices vs
        # vectors), as a decay-exempt bias/norm group is usually set up
        params = list(params)
        return AdamW([{"params": [p for p in params if p.dim() >= 2]},
                      {"params": [p for p in params if p.dim() < 2], "lr": 2e-3,
                       "weight_decay": 0.0}], lr=1e-3, weight_decay=0.1)
    return AdamW(params, lr=1e-3, weight_decay=0.1)


STEPS = 3


def _fused_ddp_worker(rank, world, port, q, kind, clip, graph):
    import torch.distributed as dist

    from flodl_b200.parallel.fused import FusedDdp

    try:
        _init(rank, world, port)
        dev = torch.device("cuda", rank)
        model = _lm(dev)
        opt = _make_opt(kind, model.parameters())
        # 1 MiB buckets with a 64 KiB tail and one-shot up to 256 KiB: the
        # 0.8M-parameter model gives several buckets of both forms
        ddp = FusedDdp(model, opt, bucket_mb=1.0, tail_mb=0.0625, oneshot_kb=256,
                       timeout_s=5.0, max_grad_norm=0.5 if clip else None)
        nb = len(ddp.buckets)
        forms = {b["oneshot"] for b in ddp.buckets}
        ids = _batch(world, dev)
        mine = ids[rank * 4:(rank + 1) * 4].clone()

        def step():
            loss = model.loss(mine, mine)
            loss.backward()
            ddp.finish()
            return loss

        if graph:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                step()  # warm-up step (counts as step 1)
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                step()
            for _ in range(STEPS - 1):
                g.replay()
        else:
            for _ in range(STEPS):
                step()
        torch.cuda.synchronize()
        ddp.comm.check()
        flat = ddp.comm.data[:ddp.numel].clone()
        gathered = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(gathered, flat)
        same = all(torch.equal(gathered[0], t) for t in gathered[1:])
        shadow_ok = bool(torch.equal(ddp.comm.shadow[:ddp.numel], flat.bfloat16()))
        norm = float(ddp.grad_norm.item()) if clip else None
        if graph:
            del g
        q.put((rank, {"replicas equal": same, "shadow equals weights": shadow_ok,
                      "buckets >= 3": nb >= 3, "both forms": len(forms) == 2 or clip},
               flat.cpu().numpy(), norm, None))
        ddp.close()
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, {}, None, None, traceback.format_exc()))


def _reference(world, kind, clip):
    """Single GPU, full batch, the same number of steps."""
    dev = torch.device("cuda", 0)
    model = _lm(dev)
    opt = _make_opt(kind, model.parameters())
    ids = _batch(world, dev)
    norm = None
    for _ in range(STEPS):
        loss = model.loss(ids, ids)
        loss.backward()
        if clip:
            grads = [p.grad for p in model.parameters() if p.grad is not None]
            norm = float(torch.linalg.vector_norm(torch.stack(
                [torch.linalg.vector_norm(g.float()) for g in grads])))
            if norm > 0.5:
                for gr in grads:
                    gr.mul_(0.5 / (norm + 1e-6))
        opt.step()
        opt.zero_grad()
    return torch.cat([g.arena.data for g in opt.groups]).cpu(), norm


@pytest.mark.parametrize("world", WORLDS)
@pytest.mark.parametrize("kind,clip,graph", [("adamw", False, False), ("sgd", False, False),
                                             ("adamw", True, False), ("adamw", False, True),
                                             ("adamw2", False, False)])
def test_fused_ddp_matches_single_gpu_full_batch(world, kind, clip, graph):
    _need_gpus(world)
    res = _spawn(_fused_ddp_worker, world, kind, clip, graph)
    for rank, checks, _, _, err in res:
        assert err is None, err
        bad = [k for k, v in checks.items() if not v]
        assert not bad, f"rank {rank}: failed {bad}"
    ref, ref_norm = _reference(world, kind, clip)
    got = torch.from_numpy(res[0][2])[:ref.numel()]
    if kind == "adamw2":
        # AdamW moves an element with a near-zero gradient by up to lr per step
        # whatever the gradient's size, so reduction-order noise can flip such
        # an element's steps: a few dozen of the second group's bias / norm
        # elements (lr 2e-3, no decay; measured up to 14 at 4 GPUs) may differ
        # by up to 2 lr per step, the rest must agree as in the other cases (a
        # wrong bucket or group boundary would break thousands)
        diff = (got - ref).abs()
        loose = diff > 2e-3 + 2e-2 * ref.abs()
        assert int(loose.sum()) <= 48, int(loose.sum())
        assert float(diff.max()) <= 2 * 2e-3 * STEPS + 1e-6, float(diff.max())
    else:
        torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-3)
    if clip:
        got_norm = res[0][3]
        assert abs(got_norm - ref_norm) <= 0.03 * ref_norm, (got_norm, ref_norm)
