"""Numerics of the sm_100a kernels against plain fp32 PyTorch references."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _C():
    from flodl_b200._ext import cuda_ext
    return cuda_ext()


@pytest.mark.parametrize("C,dtype", [(512, torch.float32), (768, torch.float32), (64, torch.bfloat16), (1000, torch.float32)])
def test_layernorm_fwd_bwd(C, dtype):
    torch.manual_seed(0)
    from flodl_b200.ops.norm import layer_norm
    R = 1000
    x = torch.randn(R, C, device="cuda").to(dtype).requires_grad_()
    w = torch.randn(C, device="cuda").requires_grad_()
    b = torch.randn(C, device="cuda").requires_grad_()
    y = layer_norm(x, w, b, 1e-5, out_bf16=False)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().clone().requires_grad_()
    br = b.detach().clone().requires_grad_()
    yr = F.layer_norm(xr, (C,), wr, br, 1e-5)
    yr.backward(dy.float())
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-4
    torch.testing.assert_close(y.float(), yr, rtol=tol, atol=tol)
    # dy is rounded to bf16 inside the kernel
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(w.grad, wr.grad, rtol=3e-2, atol=3e-1)
    torch.testing.assert_close(b.grad, br.grad, rtol=3e-2, atol=3e-1)


def test_ln_bwd_fused_extras():
    torch.manual_seed(1)
    C = _C()
    R, Cd = 512, 512
    x = torch.randn(R, Cd, device="cuda")
    w = torch.randn(Cd, device="cuda")
    mean = torch.empty(R, device="cuda"); rstd = torch.empty(R, device="cuda")
    y = torch.empty(R, Cd, device="cuda", dtype=torch.bfloat16)
    C.ln_fwd(x, w, None, y, None, mean, rstd, 1e-5)
    dy = torch.randn(R, Cd, device="cuda").bfloat16()
    dres = torch.randn(R, Cd, device="cuda")
    dx = torch.empty(R, Cd, device="cuda"); dx16 = torch.empty(R, Cd, device="cuda", dtype=torch.bfloat16)
    colsum = torch.zeros(Cd, device="cuda")
    C.ln_bwd(dy, x, mean, rstd, w, dres, dx, dx16, None, None, colsum)
    xr = x.clone().requires_grad_()
    yr = F.layer_norm(xr, (Cd,), w, None, 1e-5)
    yr.backward(dy.float())
    ref = xr.grad + dres
    torch.testing.assert_close(dx, ref, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(dx16.float(), ref, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(colsum, ref.sum(0), rtol=1e-3, atol=1e-2)


@pytest.mark.parametrize("V,smooth,ignore", [(256, 0.0, False), (30522, 0.1, True), (10, 0.0, False),
                                             (1000, 0.1, True), (2048, 0.0, True), (520, 0.0, False)])
def test_softmax_ce(V, smooth, ignore):
    torch.manual_seed(2)
    from flodl_b200.ops.loss import cross_entropy
    T = 777
    logits = (torch.randn(T, V, device="cuda") * 3).bfloat16().requires_grad_()
    tgt = torch.randint(0, V, (T,), device="cuda")
    if ignore:
        tgt[::3] = -100
    loss = cross_entropy(logits, tgt, ignore_index=-100, label_smoothing=smooth)
    loss.backward()
    lr = logits.detach().float().requires_grad_()
    ref = F.cross_entropy(lr, tgt, ignore_index=-100, label_smoothing=smooth)
    ref.backward()
    torch.testing.assert_close(loss, ref, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(logits.grad.float(), lr.grad, rtol=2e-2, atol=2e-5)


def _attn_ref(qkv, B, S, H, causal, key_pad=None):
    D = qkv.shape[1] // (3 * H)
    q, k, v = qkv.float().view(B, S, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(D)
    if causal:
        s = s.masked_fill(~torch.ones(S, S, dtype=torch.bool, device=qkv.device).tril(), float("-inf"))
    if key_pad is not None:
        s = s.masked_fill(key_pad[:, None, None, :], float("-inf"))
    p = s.softmax(-1)
    return (p @ v).permute(0, 2, 1, 3).reshape(B * S, H * D)


@pytest.mark.parametrize("B,S,H,causal", [(2, 256, 2, True), (2, 256, 2, False), (1, 200, 3, True), (2, 512, 2, False), (1, 384, 1, True)])
def test_flash_attention_fwd_bwd(B, S, H, causal):
    torch.manual_seed(3)
    from flodl_b200.ops.attention import attention_packed
    D = 64
    qkv = torch.randn(B * S, 3 * H * D, device="cuda").bfloat16().requires_grad_()
    out = attention_packed(qkv, B, S, H, causal)
    dout = torch.randn_like(out)
    out.backward(dout)
    qr = qkv.detach().float().requires_grad_()
    ref = _attn_ref(qr, B, S, H, causal)
    ref.backward(dout.float())
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(qkv.grad.float(), qr.grad, rtol=5e-2, atol=5e-2)


@pytest.mark.parametrize("kind", ["suffix", "scattered"])
def test_flash_attention_padding_mask(kind):
    """Right padding (taken as a shorter row limit per key tile) and padding
    scattered through the keys (the per-key mask)."""
    torch.manual_seed(4)
    from flodl_b200.ops.attention import attention_packed
    B, S, H, D = 2, 256, 2, 64
    qkv = torch.randn(B * S, 3 * H * D, device="cuda").bfloat16().requires_grad_()
    pad = torch.zeros(B, S, dtype=torch.bool, device="cuda")
    if kind == "suffix":
        pad[0, 200:] = True
        pad[1, 17:] = True
    else:
        pad[0, 40:90] = True
        pad[0, 130:131] = True
        pad[1] = torch.rand(S, device="cuda") < 0.3
        pad[1, 0] = False
    out = attention_packed(qkv, B, S, H, False, pad)
    dout = torch.randn_like(out)
    out.backward(dout)
    qr = qkv.detach().float().requires_grad_()
    ref = _attn_ref(qr, B, S, H, False, pad)
    ref.backward(dout.float())
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(qkv.grad.float(), qr.grad, rtol=5e-2, atol=5e-2)


def _attn_ref_chunked(qkv, dout, B, S, H, causal, key_pad=None, chunk=8):
    """fp32 attention output and input gradient, computed batch chunk by batch
    chunk so the [B, H, S, S] score tensors stay small."""
    outs, grads = [], []
    for b0 in range(0, B, chunk):
        b1 = min(B, b0 + chunk)
        q = qkv[b0 * S:b1 * S].detach().float().requires_grad_()
        kp = None if key_pad is None else key_pad[b0:b1]
        o = _attn_ref(q, b1 - b0, S, H, causal, kp)
        o.backward(dout[b0 * S:b1 * S].float())
        outs.append(o.detach())
        grads.append(q.grad)
    return torch.cat(outs), torch.cat(grads)


@pytest.mark.parametrize("B,S,H,causal,padded", [(64, 256, 8, True, False), (32, 512, 12, False, True)])
def test_flash_attention_production_shapes(B, S, H, causal, padded):
    """The LM (B64 H8 S256 causal) and BERT (B32 H12 S512, padding mask) shapes:
    hundreds of work items per launch, so every CTA of the persistent kernels
    walks several items (item-parity buffers, next-item K/V prefetch and the
    heaviest-first order all run)."""
    torch.manual_seed(11)
    from flodl_b200.ops.attention import attention_packed
    D = 64
    items = B * H * ((S + 127) // 128)
    assert items >= 2 * torch.cuda.get_device_properties(0).multi_processor_count
    qkv = torch.randn(B * S, 3 * H * D, device="cuda").bfloat16().requires_grad_()
    pad = None
    if padded:
        lens = torch.randint(S // 4, S + 1, (B,), device="cuda")
        lens[0] = S
        pad = torch.arange(S, device="cuda")[None, :] >= lens[:, None]
    out = attention_packed(qkv, B, S, H, causal, pad)
    dout = torch.randn_like(out)
    out.backward(dout)
    ref_out, ref_grad = _attn_ref_chunked(qkv, dout, B, S, H, causal, pad)
    torch.testing.assert_close(out.float(), ref_out, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(qkv.grad.float(), ref_grad, rtol=5e-2, atol=5e-2)


def test_softmax_ce_out_of_range_target_reports_error():
    """A target outside [0, V) is skipped (never read as an index) and recorded
    as kErrBadLabel (4) in the kernel error word."""
    torch.manual_seed(12)
    C = _C()
    from flodl_b200.ops.loss import cross_entropy
    T, V = 300, 50
    logits = torch.randn(T, V, device="cuda").bfloat16()
    tgt = torch.randint(0, V, (T,), device="cuda")
    tgt[5] = V
    tgt[T - 1] = 1 << 40
    torch.cuda.synchronize()
    C.clear_kernel_error()
    loss = cross_entropy(logits, tgt)
    torch.cuda.synchronize()
    assert C.kernel_error() == 4
    C.clear_kernel_error()
    ref_t = tgt.clone()
    ref_t[[5, T - 1]] = -100
    ref = F.cross_entropy(logits.float(), ref_t, ignore_index=-100)
    torch.testing.assert_close(loss, ref, rtol=1e-4, atol=1e-4)
    cross_entropy(logits, ref_t)
    torch.cuda.synchronize()
    assert C.kernel_error() == 0


def test_adamw_kernel_matches_torch():
    torch.manual_seed(5)
    C = _C()
    n = 10007
    p = torch.randn(n, device="cuda"); g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda"); v = torch.zeros(n, device="cuda")
    sh = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    lr = torch.tensor(1e-3, device="cuda"); step = torch.tensor(0.0, device="cuda")
    pr = p.clone().requires_grad_()
    opt = torch.optim.AdamW([pr], lr=1e-3, weight_decay=0.1)
    for _ in range(3):
        C.add_scalar(step, 1.0)
        C.adamw(p, g, m, v, sh, lr, step, None, 0.9, 0.999, 1e-8, 0.1, True, False)
        pr.grad = g.clone()
        opt.step()
    torch.testing.assert_close(p, pr.detach(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(sh.float(), p, rtol=1e-2, atol=1e-2)


def test_sgd_kernel_matches_torch():
    torch.manual_seed(6)
    C = _C()
    n = 4099
    p = torch.randn(n, device="cuda"); buf = torch.zeros(n, device="cuda")
    lr = torch.tensor(0.1, device="cuda")
    pr = p.clone().requires_grad_()
    opt = torch.optim.SGD([pr], lr=0.1, momentum=0.9, weight_decay=5e-4)
    for i in range(3):
        g = torch.randn(n, device="cuda")
        first = torch.tensor(1.0 if i == 0 else 0.0, device="cuda")
        C.sgd(p, g, buf, None, lr, None, first, 0.9, 0.0, 5e-4, False, False)
        pr.grad = g.clone()
        opt.step()
    torch.testing.assert_close(p, pr.detach(), rtol=1e-5, atol=1e-6)


@pytest.fixture
def fused_linear_only():
    """Route even small problems through the tcgen05 kernels."""
    import importlib
    L = importlib.import_module("flodl_b200.ops.linear")  # the module, not the function
    L.set_small_gemm_tiles(0)
    yield
    L.set_small_gemm_tiles(None)


def test_linear_small_problem_library_path_matches():
    torch.manual_seed(5)
    from flodl_b200.ops.linear import linear
    x = torch.randn(256, 1024, device="cuda").requires_grad_()
    w = (torch.randn(1024, 1024, device="cuda") * 0.03).requires_grad_()
    b = torch.randn(1024, device="cuda").requires_grad_()
    y = linear(x, w, b, act="gelu")
    y.float().sum().backward()
    xr, wr, br = [t.detach().clone().requires_grad_() for t in (x, w, b)]
    yr = F.gelu(F.linear(xr.bfloat16().float(), wr.bfloat16().float(), br))
    yr.sum().backward()
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    for got, ref in ((x.grad, xr.grad), (w.grad, wr.grad), (b.grad, br.grad)):
        assert ((got - ref).norm() / ref.norm()).item() < 2e-2


def test_linear_op_fwd_bwd_gelu_residual(fused_linear_only):
    torch.manual_seed(7)
    from flodl_b200.ops.linear import linear
    x = torch.randn(300, 256, device="cuda").requires_grad_()
    w = (torch.randn(512, 256, device="cuda") * 0.05).requires_grad_()
    b = torch.randn(512, device="cuda").requires_grad_()
    res = torch.randn(300, 512, device="cuda").requires_grad_()
    y = linear(x, w, b, act="gelu", residual=res)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr, wr, br, rr = [t.detach().clone().requires_grad_() for t in (x, w, b, res)]
    yr = rr + F.gelu(F.linear(xr.bfloat16().float(), wr.bfloat16().float(), br))
    yr.backward(dy)
    torch.testing.assert_close(y, yr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad, xr.grad, rtol=3e-2, atol=3e-2)
    # the GELU-backward operand of the weight-gradient GEMM is bf16, so a few
    # elements of a 300-row reduction differ by more than a pointwise bound;
    # compare the whole tensor by relative Frobenius error instead
    for got, ref in ((w.grad, wr.grad), (b.grad, br.grad)):
        rel = ((got - ref).norm() / ref.norm()).item()
        assert rel < 1e-2, rel
    torch.testing.assert_close(res.grad, rr.grad)


def test_gelu_epilogue_math_matches_erf_gelu():
    """The epilogue GELU (erf after Abramowitz & Stegun 7.1.28) against
    PyTorch's erf GELU and its derivative, on a dense grid."""
    from flodl_b200._ext import cuda_ext
    x = torch.linspace(-12, 12, 1 << 20, device="cuda", dtype=torch.float64)
    xf = x.float().contiguous()
    y = torch.empty_like(xf)
    d = torch.empty_like(xf)
    cuda_ext().gelu_eval_f32(xf, y, d)
    ref = F.gelu(xf.double())
    cdf = 0.5 * (1 + torch.erf(xf.double() / 2 ** 0.5))
    dref = cdf + xf.double() * torch.exp(-0.5 * xf.double() ** 2) / (2 * torch.pi) ** 0.5
    err = (y.double() - ref).abs() / (1 + xf.double().abs())
    assert err.max().item() < 2e-6, err.max().item()
    derr = (d.double() - dref).abs()
    assert derr.max().item() < 2e-6, derr.max().item()


def test_linear_odd_features_padded_path(fused_linear_only):
    torch.manual_seed(11)
    from flodl_b200.ops.linear import linear
    x = torch.randn(37, 20, device="cuda").requires_grad_()
    w = (torch.randn(10, 20, device="cuda") * 0.2).requires_grad_()
    b = torch.randn(10, device="cuda").requires_grad_()
    y = linear(x, w, b)
    dy = torch.randn_like(y.float())
    y.float().backward(dy)
    xr, wr, br = [t.detach().clone().requires_grad_() for t in (x, w, b)]
    yr = F.linear(xr.bfloat16().float(), wr.bfloat16().float(), br)
    yr.backward(dy)
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    for got, ref in ((x.grad, xr.grad), (w.grad, wr.grad), (b.grad, br.grad)):
        assert ((got - ref).norm() / ref.norm()).item() < 2e-2


def test_flash_attention_previous_kernels_still_match():
    """FLODL_FLASH_FWD=v1 / FLODL_FLASH_BWD=v1 select the one-CTA-per-SM
    forward and the key-tile backward with the f32 dQ accumulator (kept for
    comparison runs); checked in a child process because the switches are read
    once per process."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys\n"
        "sys.path.insert(0, %r)\n"
        "from tests.test_kernels_gpu import test_flash_attention_fwd_bwd as t\n"
        "t(2, 256, 2, True); t(1, 200, 3, False)\n"
        "print('ok')\n" % root)
    env = dict(os.environ, FLODL_FLASH_FWD="v1", FLODL_FLASH_BWD="v1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=300, cwd=root)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


@pytest.mark.parametrize("C,dtype", [(512, torch.float32), (1000, torch.float32),
                                     (4096, torch.bfloat16), (768, torch.bfloat16)])
def test_rms_norm_kernel_matches_fp32(C, dtype):
    """RMSNorm forward/backward kernels (weight gradient included) against
    the fp32 composition of the reference formula."""
    from flodl_b200.ops import rms_norm
    torch.manual_seed(7)
    rows = 333
    x = (torch.randn(rows, C, device="cuda") * 1.5 + 0.2).to(dtype).requires_grad_()
    w = (torch.rand(C, device="cuda") + 0.5).requires_grad_()
    y = rms_norm(x, w, 1e-5)
    assert y.dtype == dtype
    dy = torch.randn(rows, C, device="cuda").to(dtype)
    y.backward(dy)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().clone().requires_grad_()
    ref = xr / torch.sqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * wr
    ref.backward(dy.float())
    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(y.float(), ref, **tol)
    torch.testing.assert_close(x.grad.float(), xr.grad, **tol)
    torch.testing.assert_close(w.grad, wr.grad, rtol=2e-3 if dtype == torch.float32 else 3e-2,
                               atol=2e-3 if dtype == torch.float32 else 0.5)


@pytest.mark.parametrize("D,masked", [(64, False), (64, True), (128, False)])
def test_sdpa_routes_and_matches_torch(D, masked):
    """Functional SDPA: head size 64 with no mask or a key-padding mask runs
    the flash kernel, other head sizes the composed form; both match torch's
    fp32 attention."""
    from flodl_b200.ops.attention import scaled_dot_product_attention as sdpa
    torch.manual_seed(11)
    B, H, S = 2, 3, 200
    q, k, v = (torch.randn(B, H, S, D, device="cuda") for _ in range(3))
    mask = None
    if masked:
        mask = torch.ones(B, 1, 1, S, dtype=torch.bool, device="cuda")
        mask[0, ..., 150:] = False
        mask[1, ..., 37:] = False
    out = sdpa(q, k, v, attn_mask=mask)
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    torch.testing.assert_close(out.float(), ref, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("V", [256, 100])
def test_onehot_and_position_gradient_kernels(V):
    """One-hot rows of the embedding-gradient GEMM (16-byte stores when V is
    a multiple of 8, element stores otherwise) and the position-table
    gradient (a sum over the batch)."""
    from flodl_b200._ext import cuda_ext
    C = cuda_ext()
    torch.manual_seed(5)
    T = 1000
    ids = torch.randint(0, V, (T,), device="cuda")
    oh = torch.full((T, V), 7.0, device="cuda", dtype=torch.bfloat16)
    C.onehot_bf16(ids, oh)
    torch.testing.assert_close(oh.float(), torch.nn.functional.one_hot(ids, V).float())
    B, S, D = 5, 37, 64
    dy = torch.randn(B, S, D, device="cuda")
    dpos = torch.ones(S, D, device="cuda")
    C.pos_grad(dy, dpos, B, S)
    torch.testing.assert_close(dpos, 1.0 + dy.sum(0), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("N,C,HW,G,dtype", [(4, 32, 64, 8, torch.float32),
                                            (3, 48, 17 * 9, 6, torch.float32),
                                            (2, 64, 256, 32, torch.bfloat16),
                                            (2, 16, 1024, 2, torch.float32)])
def test_group_norm_kernel_matches_fp32(N, C, HW, G, dtype):
    """GroupNorm forward/backward kernels (affine gradients included) against
    PyTorch's fp32 group_norm."""
    from flodl_b200.ops import group_norm
    torch.manual_seed(9)
    x = (torch.randn(N, C, HW, device="cuda") * 2 + 0.3).to(dtype).requires_grad_()
    w = (torch.rand(C, device="cuda") + 0.5).requires_grad_()
    b = torch.randn(C, device="cuda").requires_grad_()
    y = group_norm(x, G, w, b, 1e-5)
    dy = torch.randn(N, C, HW, device="cuda").to(dtype)
    y.backward(dy)
    xr = x.detach().float().requires_grad_()
    wr, br = w.detach().clone().requires_grad_(), b.detach().clone().requires_grad_()
    ref = torch.nn.functional.group_norm(xr, G, wr, br, 1e-5)
    ref.backward(dy.float())
    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(y.float(), ref, **tol)
    torch.testing.assert_close(x.grad.float(), xr.grad, **tol)
    gt = dict(rtol=1e-3, atol=1e-3) if dtype == torch.float32 else dict(rtol=3e-2, atol=0.3)
    torch.testing.assert_close(w.grad, wr.grad, **gt)
    torch.testing.assert_close(b.grad, br.grad, **gt)


@pytest.mark.parametrize("shape,k,s,p,d,ceil,dtype", [
    ((2, 3, 28, 28), 2, 2, 0, 1, False, torch.float32),
    ((2, 4, 17, 13), 3, 2, 1, 1, True, torch.float32),
    ((1, 8, 16, 16), 3, 1, 1, 2, False, torch.bfloat16),
])
def test_max_pool2d_kernel_matches_torch(shape, k, s, p, d, ceil, dtype):
    """Max pooling forward (values) and backward (gradient routed to each
    window's maximum) against PyTorch's."""
    from flodl_b200.ops import max_pool1d, max_pool2d
    torch.manual_seed(2)
    x = torch.randn(*shape, device="cuda").to(dtype).requires_grad_()
    y = max_pool2d(x, k, s, p, d, ceil)
    xr = x.detach().clone().requires_grad_()
    yr = torch.nn.functional.max_pool2d(xr, k, s, p, d, ceil)
    assert y.shape == yr.shape
    torch.testing.assert_close(y, yr)
    dy = torch.randn_like(yr)
    y.backward(dy)
    # reference gradient in fp32 (bf16 gradients accumulate overlapping windows
    # with bf16 atomic adds: a few ulps per overlap)
    xf = x.detach().float().requires_grad_()
    torch.nn.functional.max_pool2d(xf, k, s, p, d, ceil).backward(dy.float())
    tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=5e-2, atol=5e-2)
    torch.testing.assert_close(x.grad.float(), xf.grad, **tol)
    x1 = torch.randn(3, 5, 40, device="cuda")
    torch.testing.assert_close(max_pool1d(x1, 3, 2, 1), torch.nn.functional.max_pool1d(x1, 3, 2, 1))


@pytest.mark.parametrize("dtype,p", [(torch.float32, 0.1), (torch.float32, 0.5),
                                     (torch.bfloat16, 0.3)])
def test_dropout_kernel_mask_scale_and_backward(dtype, p):
    """Dropout kernel: the kept fraction is 1 - p, kept values are scaled by
    1/(1-p), the backward applies the forward's mask (regenerated from the
    same seed and offset), and two calls draw different masks."""
    from flodl_b200.ops import dropout
    torch.manual_seed(12)
    n = 1 << 20
    x = (torch.rand(n, device="cuda") + 0.5).to(dtype).requires_grad_()
    y = dropout(x, p, True)
    kept = y != 0
    frac = kept.float().mean().item()
    assert abs(frac - (1 - p)) < 5e-3, frac
    torch.testing.assert_close(y[kept].float(), (x[kept].float() / (1 - p)).to(dtype).float(),
                               rtol=1e-2 if dtype == torch.bfloat16 else 1e-6, atol=0)
    dy = torch.ones_like(y)
    y.backward(dy)
    assert torch.equal(x.grad != 0, kept)
    y2 = dropout(x.detach(), p, True)
    assert not torch.equal(y2 != 0, kept)
    assert torch.equal(dropout(x.detach(), p, False), x.detach())
