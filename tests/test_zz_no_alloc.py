"""The allocation-free softmax cross-entropy C entry point.

Called through its exported C symbol (as a caller that cannot allocate would
call it) and compared with the regular kernel entry point on two calls in a
row, which also checks that the shared fixed scratch array carries no state
from one call into the next.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from flodl_b200._ext import cuda_ext
    lib = ctypes.CDLL(cuda_ext().__file__)
    fn = lib.flodl_softmax_ce_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.flodl_softmax_ce_noalloc_max_rows.restype = ctypes.c_int
    lib.flodl_softmax_ce_noalloc_bad_rows.restype = ctypes.c_int
    lib.flodl_softmax_ce_noalloc_bad_rows.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    return lib, fn


def _regular(logits, tgt, smoothing):
    from flodl_b200._ext import cuda_ext
    loss = torch.zeros((), device="cuda")
    inv = torch.empty((), device="cuda")
    dl = torch.empty_like(logits)
    cuda_ext().softmax_ce(logits, tgt, loss, inv, dl, -100, smoothing)
    return loss, dl


def _noalloc(fn, logits, tgt, smoothing, loss, dl):
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(logits.data_ptr(), logits.stride(0), tgt.data_ptr(), logits.shape[0], logits.shape[1],
            -100, smoothing, loss.data_ptr(), dl.data_ptr(), stream)
    assert rc == 0, f"flodl_softmax_ce_noalloc returned {rc}"


@pytest.mark.parametrize("T,V,smoothing", [(4096, 256, 0.0), (1000, 30522, 0.1)])
def test_noalloc_matches_regular_entry_point_twice(T, V, smoothing):
    lib, fn = _lib()
    torch.manual_seed(0)
    for call in range(2):
        logits = (torch.randn(T, V, device="cuda") * (2 + call)).bfloat16()
        tgt = torch.randint(0, V, (T,), device="cuda")
        tgt[call::5] = -100
        ref_loss, ref_dl = _regular(logits, tgt, smoothing)
        loss = torch.full((), float("nan"), device="cuda")
        dl = torch.full_like(logits, float("nan"))
        _noalloc(fn, logits, tgt, smoothing, loss, dl)
        torch.cuda.synchronize()
        torch.testing.assert_close(loss, ref_loss, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(dl.float(), ref_dl.float(), rtol=2e-2, atol=2e-5)


def test_noalloc_rejects_oversize():
    lib, fn = _lib()
    cap = lib.flodl_softmax_ce_noalloc_max_rows()
    rows = cap + 1
    logits = torch.zeros(rows, 1, device="cuda", dtype=torch.bfloat16)
    tgt = torch.zeros(rows, device="cuda", dtype=torch.int64)
    loss = torch.zeros((), device="cuda")
    rc = fn(logits.data_ptr(), 1, tgt.data_ptr(), rows, 1, -100, 0.0, loss.data_ptr(), None,
            torch.cuda.current_stream().cuda_stream)
    assert rc == -1


def test_noalloc_out_of_range_targets_are_skipped_and_counted():
    """A target outside [0, V) is never used as an index: the row counts as
    ignored (loss and gradient match the regular entry point with that target
    set to ignore_index) and the bad-row count reports it."""
    lib, fn = _lib()
    T, V = 512, 256
    torch.manual_seed(1)
    logits = torch.randn(T, V, device="cuda").bfloat16()
    tgt = torch.randint(0, V, (T,), device="cuda")
    tgt[3] = V          # one past the row
    tgt[T - 1] = 10 * V  # the last row: far past the end of the logits buffer
    tgt[7] = -5
    tgt[11] = -100       # ignore_index: not a bad row
    ref_t = tgt.clone()
    ref_t[[3, T - 1, 7]] = -100
    ref_loss, ref_dl = _regular(logits, ref_t, 0.0)
    loss = torch.full((), float("nan"), device="cuda")
    dl = torch.full_like(logits, float("nan"))
    _noalloc(fn, logits, tgt, 0.0, loss, dl)
    bad = ctypes.c_int(-1)
    rc = lib.flodl_softmax_ce_noalloc_bad_rows(torch.cuda.current_stream().cuda_stream,
                                               ctypes.byref(bad))
    assert rc == 0
    assert bad.value == 3
    torch.testing.assert_close(loss, ref_loss, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(dl.float(), ref_dl.float(), rtol=2e-2, atol=2e-5)
    # a following call with valid targets reports no bad rows
    _noalloc(fn, logits, ref_t, 0.0, loss, dl)
    rc = lib.flodl_softmax_ce_noalloc_bad_rows(torch.cuda.current_stream().cuda_stream,
                                               ctypes.byref(bad))
    assert rc == 0 and bad.value == 0
