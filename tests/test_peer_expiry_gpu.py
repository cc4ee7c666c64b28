"""Bounded peer waits on one GPU: a communicator whose "peer" never launches.

The peer regions of rank 1 are a second allocation on the same GPU that no
kernel ever touches, so rank 0's start meeting can never complete. Its waits
must give up after the communicator's limit (50 ms here), record the peer
timeout in the host-mapped error word and return; ``PeerComm.check`` must turn
that into ``PeerTimeout``; a fresh communicator must work afterwards (the GPU
context stays usable). Only one kernel runs at a time and nothing waits on
another kernel, so nothing here can hang.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ghost_regions(C, numel):
    ptrs = {}
    for name, nbytes in (("data", numel * 4), ("grad", numel * 4), ("shadow", numel * 2),
                         ("sig", C.signal_words() * 4)):
        ptrs[name] = C.peer_alloc(nbytes)[0]
    return ptrs


@pytest.mark.parametrize("op", ["all_reduce", "broadcast", "weighted_average"])
def test_peer_wait_expires_and_reports(op):
    from flodl_b200._ext import cuda_ext
    from flodl_b200.parallel.peer import PeerComm, PeerTimeout

    C = cuda_ext()
    dev = torch.device("cuda", 0)
    n = 1 << 16
    comm = PeerComm(n, dev, timeout_s=0.05)
    ghost = _ghost_regions(C, comm.numel)
    comm.world = 2  # rank 0 of a two-rank communicator whose rank 1 never shows up
    for name in ("data", "grad", "shadow", "sig"):
        comm.ptrs[name] = [comm.ptrs[name][0], ghost[name]]
    t0 = time.monotonic()
    if op == "all_reduce":
        comm.all_reduce_(n, slot=3)
    elif op == "broadcast":
        comm.broadcast_(n, root=1, slot=3)
    else:
        comm.weighted_average_(n, 1.0, slot=3, div=torch.zeros(2, device=dev))
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    assert elapsed < 5.0, f"the bounded wait took {elapsed:.2f} s"
    with pytest.raises(PeerTimeout):
        comm.check()
    assert int(comm.err_host[0].item()) == 2  # kErrPeerTimeout
    comm.close()
    for p in ghost.values():
        C.peer_free(p)

    # a fresh communicator on the same GPU works
    fresh = PeerComm(n, dev, timeout_s=1.0)
    x = torch.randn(n, device=dev)
    fresh.grad[:n].copy_(x)
    fresh.all_reduce_(n, average=False, slot=0)
    torch.cuda.synchronize()
    fresh.check()
    assert torch.equal(fresh.grad[:n], x)
    fresh.close()
