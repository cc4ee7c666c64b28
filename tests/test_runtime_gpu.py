"""GPU runtime wrappers and the single-process NCCL group on CUDA."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_stream_guard_events_and_memory_stats():
    from flodl_b200.utils import cuda as C
    assert C.gpu_available() and C.device_count() >= 1 and C.arch(0) == "sm_100"
    s = C.stream_from_pool(0)
    before = torch.cuda.current_stream()
    with C.StreamGuard(s):
        assert torch.cuda.current_stream() == s
        a, b = C.CudaEvent().record(), None
        x = torch.randn(1024, 1024, device="cuda") @ torch.randn(1024, 1024, device="cuda")
        b = C.CudaEvent().record()
    assert torch.cuda.current_stream() == before
    b.synchronize()
    assert a.elapsed_ms(b) >= 0.0 and x.shape == (1024, 1024)
    st = C.memory_stats(0)
    assert st["total"] > 100 * 2 ** 30 and st["peak_allocated"] >= st["allocated"]


def test_single_process_group_all_reduce_and_broadcast():
    from flodl_b200.parallel.nccl import NcclComms, ReduceOp
    n = torch.cuda.device_count()
    comms = NcclComms(list(range(n)))
    ts = [torch.full((1000,), float(i + 1), device=f"cuda:{i}") for i in range(n)]
    comms.all_reduce(ts, ReduceOp.Sum)
    assert all(torch.all(t == n * (n + 1) / 2) for t in ts)
    bs = [torch.full((10,), float(i), device=f"cuda:{i}") for i in range(n)]
    comms.broadcast(bs, root=0)
    assert all(torch.all(b == 0) for b in bs)
    assert NcclComms.version()


def test_captured_training_step_matches_eager():
    """A FlowBuilder model's whole training step (forward, loss, backward,
    fused Adam) captured as a CUDA graph follows the eager loss trajectory."""
    from flodl_b200.graph import FlowBuilder
    from flodl_b200.nn import GELU, LayerNorm, Linear
    from flodl_b200.optim import Adam
    from flodl_b200.train import StepRunner

    def make():
        torch.manual_seed(0)
        g = (FlowBuilder.from_(Linear(256, 512, device="cuda")).through(GELU())
             .through(LayerNorm(512, device="cuda")).also(Linear(512, 512, device="cuda"))
             .through(Linear(512, 256, device="cuda")).build())
        return g, Adam(g.parameters(), lr=1e-3)

    gen = torch.Generator(device="cuda").manual_seed(1)
    batches = [(torch.randn(1024, 256, device="cuda", generator=gen),
                torch.randn(1024, 256, device="cuda", generator=gen)) for _ in range(8)]
    lf = lambda out, y: torch.nn.functional.mse_loss(out.float(), y)
    g1, o1 = make()
    eager = []
    for _ in range(3):  # the capture's warm-up steps run on the first batch
        l = lf(g1(batches[0][0]), batches[0][1]); l.backward(); o1.step(); o1.zero_grad()
    for x, y in batches:
        l = lf(g1(x), y); l.backward(); o1.step(); o1.zero_grad()
        eager.append(l.item())
    g2, o2 = make()
    r = StepRunner.capture_training(g2, o2, lf, list(batches[0]))
    cap = [r.replay(x, y).item() for x, y in batches]
    torch.testing.assert_close(torch.tensor(cap), torch.tensor(eager), rtol=2e-2, atol=2e-3)
    # the batches are independent noise; on one fixed batch the captured step must learn
    fixed = [r.replay(*batches[0]).item() for _ in range(20)]
    assert fixed[-1] < fixed[0]


def test_captured_training_step_with_loop():
    """A for-loop graph (shared body weights, per-iteration traces kept) is
    capturable and follows the eager trajectory."""
    from flodl_b200.graph import FlowBuilder
    from flodl_b200.nn import GELU, LayerNorm, Linear
    from flodl_b200.optim import Adam
    from flodl_b200.train import StepRunner

    def make():
        torch.manual_seed(0)
        body = FlowBuilder.new().also(FlowBuilder.from_(Linear(256, 256, device="cuda"))
                                      .through(GELU()).through(LayerNorm(256, device="cuda")).build()).build()
        g = (FlowBuilder.from_(Linear(256, 256, device="cuda")).loop_body(body).for_n(4)
             .through(Linear(256, 256, device="cuda")).build())
        return g, Adam(g.parameters(), lr=1e-3)

    gen = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(64, 256, device="cuda", generator=gen)
    y = torch.randn(64, 256, device="cuda", generator=gen)
    lf = lambda out, t: torch.nn.functional.mse_loss(out.float(), t)
    g1, o1 = make()
    eager = []
    for _ in range(3 + 6):
        l = lf(g1(x), y); l.backward(); o1.step(); o1.zero_grad()
        eager.append(l.item())
    g2, o2 = make()
    r = StepRunner.capture_training(g2, o2, lf, [x, y])
    cap = [r.replay(x, y).item() for _ in range(6)]
    torch.testing.assert_close(torch.tensor(cap), torch.tensor(eager[3:]), rtol=2e-2, atol=2e-3)
    assert cap[-1] < cap[0]


def test_step_pipelined_reads_every_loss_one_step_late():
    """step_pipelined returns the previous step's loss; with flush() the
    sequence equals what step() reads synchronously."""
    from flodl_b200.graph import FlowBuilder
    from flodl_b200.nn import GELU, Linear
    from flodl_b200.optim import Adam
    from flodl_b200.train import StepRunner

    def make():
        torch.manual_seed(0)
        g = FlowBuilder.from_(Linear(64, 128, device="cuda")).through(GELU()).through(
            Linear(128, 64, device="cuda")).build()
        return g, Adam(g.parameters(), lr=1e-3)

    x = torch.randn(256, 64).pin_memory()
    y = torch.randn(256, 64).pin_memory()
    lf = lambda out, t: torch.nn.functional.mse_loss(out.float(), t)
    g1, o1 = make()
    r1 = StepRunner.capture_training(g1, o1, lf, [x.cuda(), y.cuda()])
    sync = [r1.step(x, y) for _ in range(6)]
    g2, o2 = make()
    r2 = StepRunner.capture_training(g2, o2, lf, [x.cuda(), y.cuda()])
    got = [r2.step_pipelined(x, y) for _ in range(6)]
    assert got[0] is None
    piped = got[1:] + [r2.flush()]
    assert r2.flush() is None
    torch.testing.assert_close(torch.tensor(piped), torch.tensor(sync), rtol=1e-5, atol=1e-6)
