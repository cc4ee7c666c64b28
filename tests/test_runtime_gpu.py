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
