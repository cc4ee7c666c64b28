"""Convolution / batch-norm kernels and the fused ResNet-20 training op
against PyTorch fp32 references (NHWC bf16 activations on the device)."""
import copy

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _C():
    from flodl_b200._ext import cuda_ext
    return cuda_ext()


@pytest.mark.parametrize("Cin,k,s,p,H", [(8, 3, 1, 1, 32), (16, 3, 2, 1, 32), (32, 1, 2, 0, 16),
                                         (64, 3, 1, 1, 8)])
def test_im2col_col2im_match_unfold_fold(Cin, k, s, p, H):
    C = _C()
    torch.manual_seed(0)
    N = 3
    x = torch.randn(N, Cin, H, H, device="cuda").bfloat16()
    xh = x.permute(0, 2, 3, 1).contiguous()
    Ho = (H + 2 * p - k) // s + 1
    K = Cin * k * k
    L = Ho * Ho
    cols = torch.full((N * L, K), 7.0, device="cuda", dtype=torch.bfloat16)
    C.im2col(xh, cols, k, s, p)
    # unfold gives columns ordered (c, kh, kw); the kernel orders them (kh, kw, c)
    ref = F.unfold(x.float(), k, padding=p, stride=s).reshape(N, Cin, k * k, L)
    ref = ref.permute(0, 3, 2, 1).reshape(N * L, K)
    torch.testing.assert_close(cols.float(), ref)
    # col2im = adjoint of im2col (sum over taps), with add and ReLU mask
    dcols = torch.randn(N * L, K, device="cuda").bfloat16()
    add = torch.randn(N, H, H, Cin, device="cuda").bfloat16()
    mask = torch.randn(N, H, H, Cin, device="cuda").bfloat16()
    dx = torch.empty(N, H, H, Cin, device="cuda", dtype=torch.bfloat16)
    C.col2im(dcols, dx, k, s, p, add, mask)
    dc = dcols.float().reshape(N, L, k * k, Cin).permute(0, 3, 2, 1).reshape(N, K, L)
    fold = F.fold(dc, (H, H), k, padding=p, stride=s).permute(0, 2, 3, 1)
    exp = (fold + add.float()) * (mask.float() > 0)
    torch.testing.assert_close(dx.float(), exp, rtol=2e-2, atol=5e-2)


@pytest.mark.parametrize("Cc", [16, 32, 64])
def test_batch_norm_kernels_match_torch(Cc):
    C = _C()
    torch.manual_seed(1)
    M = 4096 + 37
    y = (torch.randn(M, Cc, device="cuda") * 2 + 0.5).bfloat16()
    ident = torch.randn(M, Cc, device="cuda").bfloat16()
    gamma = torch.rand(Cc, device="cuda") + 0.5
    beta = torch.randn(Cc, device="cuda")
    rm, rv = torch.zeros(Cc, device="cuda"), torch.ones(Cc, device="cuda")
    ws = torch.zeros(2 * Cc + 1, device="cuda")
    mean, rstd = torch.empty(Cc, device="cuda"), torch.empty(Cc, device="cuda")
    out = torch.empty_like(y)
    for _ in range(2):  # the workspace must come back zeroed
        C.bn_stats(y, mean, rstd, rm, rv, ws, 1e-5, 0.1)
    C.bn_apply(y, mean, rstd, gamma, beta, ident, True, out)
    yf = y.float().requires_grad_()
    g_, b_ = gamma.clone().requires_grad_(), beta.clone().requires_grad_()
    rm2, rv2 = torch.zeros(Cc, device="cuda"), torch.ones(Cc, device="cuda")
    z = F.batch_norm(yf, rm2, rv2, g_, b_, True, 0.1, 1e-5)
    F.batch_norm(y.float(), rm2, rv2, None, None, True, 0.1, 1e-5)
    ref = torch.relu(z + ident.float())
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=3e-2)
    torch.testing.assert_close(rm, rm2, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(rv, rv2, rtol=1e-3, atol=1e-3)
    assert ws.abs().max().item() == 0.0
    # backward with the ReLU mask of the output and the masked gradient
    dy = torch.randn(M, Cc, device="cuda").bfloat16()
    ref.backward(dy.float())
    dg, db = torch.zeros(Cc, device="cuda"), torch.zeros(Cc, device="cuda")
    sums = torch.empty(2 * Cc, device="cuda")
    dx, dz = torch.empty_like(y), torch.empty_like(y)
    C.bn_bwd(dy, out, y, mean, rstd, gamma, dg, db, sums, ws, dx, dz)
    torch.testing.assert_close(dz.float(), dy.float() * (out.float() > 0))
    torch.testing.assert_close(dx.float(), yf.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(dg, g_.grad, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(db, b_.grad, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("Cc,k,s,p", [(16, 3, 1, 1), (32, 3, 2, 1), (64, 1, 2, 0)])
def test_col2im_with_batch_norm_sums_matches_fp32(Cc, k, s, p):
    """col2im_bn = col2im (+ add, * mask) whose output is a batch norm's output
    gradient, with that batch norm's backward sums reduced in the same pass;
    bn_bwd_apply finishes the input gradient."""
    C = _C()
    torch.manual_seed(3)
    N, H = 16, 16
    Ho = (H + 2 * p - k) // s + 1
    L, K = Ho * Ho, Cc * k * k
    M = N * H * H
    dcols = torch.randn(N * L, K, device="cuda").bfloat16()
    add = torch.randn(N, H, H, Cc, device="cuda").bfloat16()
    mask = torch.randn(N, H, H, Cc, device="cuda").bfloat16()
    y = (torch.randn(M, Cc, device="cuda") * 2 + 0.5).bfloat16()
    gamma = torch.rand(Cc, device="cuda") + 0.5
    mean = y.float().mean(0)
    rstd = torch.rsqrt(y.float().var(0, unbiased=False) + 1e-5)
    ws = torch.zeros(2 * Cc + 1, device="cuda")
    sums = torch.empty(2 * Cc, device="cuda")
    dg, db = torch.zeros(Cc, device="cuda"), torch.zeros(Cc, device="cuda")
    dz = torch.empty(N, H, H, Cc, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):  # the workspace must come back zeroed
        C.col2im_bn(dcols, dz, k, s, p, add, mask, y, mean, rstd, dg, db, sums, ws)
    assert ws.abs().max().item() == 0.0
    dx = torch.empty_like(y)
    C.bn_bwd_apply(dz.view(M, Cc), None, y, mean, rstd, gamma, sums, dx)
    # fp32 reference: fold, add, mask, then batch-norm backward
    dc = dcols.float().reshape(N, L, k * k, Cc).permute(0, 3, 2, 1).reshape(N, K, L)
    fold = F.fold(dc, (H, H), k, padding=p, stride=s).permute(0, 2, 3, 1)
    g = ((fold + add.float()) * (mask.float() > 0)).reshape(M, Cc)
    torch.testing.assert_close(dz.float().view(M, Cc), g, rtol=2e-2, atol=5e-2)
    xhat = (y.float() - mean) * rstd
    sg, sgx = g.sum(0), (g * xhat).sum(0)
    torch.testing.assert_close(sums[:Cc], sg, rtol=1e-2, atol=0.5)
    torch.testing.assert_close(sums[Cc:], sgx, rtol=1e-2, atol=0.5)
    torch.testing.assert_close(db, 2 * sg, rtol=1e-2, atol=1.0)
    torch.testing.assert_close(dg, 2 * sgx, rtol=1e-2, atol=1.0)
    ref = gamma * rstd * (g - sg / M - xhat * sgx / M)
    torch.testing.assert_close(dx.float(), ref, rtol=3e-2, atol=3e-2)


def test_resnet20_fused_batch_norm_backward_matches_separate_reduction(monkeypatch):
    """The backward with batch-norm sums reduced inside col2im deviates from
    fp32 no more than the backward with the separate reduction kernels (bf16
    ResNet gradients are ill-conditioned: any change of summation order moves
    them by percents, so the two bf16 runs are compared through fp32)."""
    import flodl_b200.ops.resnet as R
    from flodl_b200.models import ResNet20

    torch.manual_seed(0)
    cpu = ResNet20()
    m = copy.deepcopy(cpu)
    m.move_to_device(torch.device("cuda"))
    x = torch.randn(64, 3, 32, 32)
    t = torch.randint(0, 10, (64,))
    cpu.loss(x, t).backward()
    dev = []
    for fused in (False, True):
        monkeypatch.setattr(R, "FUSED_BN_BWD", fused)
        for q in m.parameters():
            q.grad = None
        m.loss(x.cuda(), t.cuda()).backward()
        torch.cuda.synchronize()
        dev.append([((q.grad.cpu() - pc.grad).norm() / pc.grad.norm()).item()
                    for q, pc in zip(m.parameters(), cpu.parameters())])
    sep, fus = dev
    for (name, _), a, b in zip(m.named_parameters(), sep, fus):
        assert b < 2.0 * a + 0.05, f"{name}: fused {b:.3f} vs separate {a:.3f}"
    assert sum(fus) < 1.25 * sum(sep) + 0.05, (sum(fus), sum(sep))


def test_resnet20_fused_matches_bf16_autocast_reference():
    """bf16 training of ResNet-20 deviates from fp32 by tens of percent per
    gradient (BatchNorm backward cancels most of each gradient); the fused op
    must deviate from fp32 no more than PyTorch's own bf16 autocast run of the
    same network does."""
    from flodl_b200.bench_support import _TorchResNet20
    from flodl_b200.models import ResNet20

    torch.manual_seed(0)
    cpu = ResNet20()
    gpu = copy.deepcopy(cpu)
    gpu.move_to_device(torch.device("cuda"))
    ref = _TorchResNet20()
    with torch.no_grad():
        for (n1, p1), (n2, p2) in zip(cpu.named_parameters(), ref.named_parameters()):
            assert p1.shape == p2.shape, (n1, n2)
            p2.copy_(p1)
    ref = ref.cuda().to(memory_format=torch.channels_last)
    x = torch.randn(32, 3, 32, 32)
    t = torch.randint(0, 10, (32,))
    lc = cpu.loss(x, t)
    lc.backward()
    lg = gpu.loss(x.cuda(), t.cuda())
    lg.backward()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        la = ref(x.cuda(), t.cuda())
    la.backward()
    torch.cuda.synchronize()
    assert abs(lg.item() - lc.item()) < 5e-2, (lg.item(), lc.item())
    tot_f, tot_a = 0.0, 0.0
    for (name, pc), (_, pg), (_, pa) in zip(cpu.named_parameters(), gpu.named_parameters(),
                                            ref.named_parameters()):
        assert pg.grad is not None, name
        rf = ((pg.grad.cpu() - pc.grad).norm() / pc.grad.norm()).item()
        ra = ((pa.grad.cpu() - pc.grad).norm() / pc.grad.norm()).item()
        assert rf < 2.0 * ra + 0.05, f"{name}: fused {rf:.3f} vs autocast {ra:.3f}"
        tot_f += rf
        tot_a += ra
    assert tot_f < 1.2 * tot_a, (tot_f, tot_a)
    gb = dict(gpu.named_buffers())
    for name, bc in cpu.named_buffers():
        torch.testing.assert_close(gb[name].cpu(), bc, rtol=2e-2, atol=2e-2)


def test_generic_conv2d_and_batchnorm_ops():
    from flodl_b200 import ops
    torch.manual_seed(3)
    x = torch.randn(4, 16, 16, 16, device="cuda", requires_grad=True)
    w = torch.randn(32, 16, 3, 3, device="cuda", requires_grad=True)
    b = torch.randn(32, device="cuda", requires_grad=True)
    y = ops.conv2d(x, w, b, 2, 1)
    y.float().sum().backward()
    x2, w2, b2 = [t.detach().clone().requires_grad_() for t in (x, w, b)]
    y2 = F.conv2d(x2.bfloat16().float(), w2.bfloat16().float(), b2, 2, 1)
    y2.sum().backward()
    for u, v in ((y.float(), y2), (x.grad, x2.grad), (w.grad, w2.grad), (b.grad, b2.grad)):
        assert ((u - v).norm() / v.norm()).item() < 1e-2
    z = torch.randn(8, 32, 8, 8, device="cuda", requires_grad=True)
    g = torch.rand(32, device="cuda", requires_grad=True)
    be = torch.randn(32, device="cuda", requires_grad=True)
    rm, rv = torch.zeros(32, device="cuda"), torch.ones(32, device="cuda")
    o = ops.batch_norm2d(z, rm, rv, g, be, True, 0.1, 1e-5)
    dy = torch.randn_like(z)
    o.float().backward(dy)
    z2, g2, be2 = [t.detach().clone().requires_grad_() for t in (z, g, be)]
    rm2, rv2 = torch.zeros(32, device="cuda"), torch.ones(32, device="cuda")
    o2 = F.batch_norm(z2.bfloat16().float(), rm2, rv2, g2, be2, True, 0.1, 1e-5)
    o2.backward(dy.bfloat16().float())
    for u, v in ((o.float(), o2), (z.grad, z2.grad), (g.grad, g2.grad), (be.grad, be2.grad)):
        assert ((u - v).norm() / v.norm()).item() < 2e-2
    torch.testing.assert_close(rm, rm2, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("kh,kw,sh,sw,ph,pw", [(3, 5, 1, 2, 1, 2), (1, 7, 1, 1, 0, 3),
                                               (5, 3, 2, 1, 2, 0)])
def test_rectangular_conv2d_matches_fp32(kh, kw, sh, sw, ph, pw):
    """Any kh x kw kernel with per-axis stride and padding on the tcgen05 path,
    against an fp32 convolution of the bf16-rounded operands."""
    from flodl_b200 import ops
    torch.manual_seed(7)
    x = torch.randn(4, 12, 20, 18, device="cuda", requires_grad=True)
    w = torch.randn(16, 12, kh, kw, device="cuda", requires_grad=True)
    b = torch.randn(16, device="cuda", requires_grad=True)
    y = ops.conv2d(x, w, b, (sh, sw), (ph, pw))
    dy = torch.randn_like(y.float())
    y.float().backward(dy)
    x2, w2, b2 = [t.detach().clone().requires_grad_() for t in (x, w, b)]
    y2 = F.conv2d(x2.bfloat16().float(), w2.bfloat16().float(), b2, (sh, sw), (ph, pw))
    y2.backward(dy.bfloat16().float())
    for u, v in ((y.float(), y2), (x.grad, x2.grad), (w.grad, w2.grad), (b.grad, b2.grad)):
        assert ((u - v).norm() / v.norm()).item() < 1e-2


def test_conv1d_layer_runs_the_kernels_and_matches_fp32():
    from flodl_b200._ext import cuda_ext
    from flodl_b200.nn import Conv1d
    torch.manual_seed(8)
    conv = Conv1d(4, 32, 5, stride=2, padding=2, device=torch.device("cuda"))
    x = torch.randn(8, 4, 200, device="cuda", requires_grad=True)
    n0 = cuda_ext().launch_count()
    y = conv(x)
    assert cuda_ext().launch_count() > n0, "Conv1d did not launch this library's kernels"
    dy = torch.randn_like(y.float())
    y.float().backward(dy)
    x2 = x.detach().clone().requires_grad_()
    w2 = conv.weight.detach().clone().requires_grad_()
    b2 = conv.bias.detach().clone().requires_grad_()
    y2 = F.conv1d(x2.bfloat16().float(), w2.bfloat16().float(), b2, 2, 2)
    y2.backward(dy.bfloat16().float())
    for u, v in ((y.float(), y2), (x.grad, x2.grad), (conv.weight.grad, w2.grad),
                 (conv.bias.grad, b2.grad)):
        assert ((u - v).norm() / v.norm()).item() < 1e-2


@pytest.mark.parametrize("k,s,p,op", [(3, 2, 1, 1), (4, 2, 1, 0), (3, 1, 1, 0)])
def test_conv_transpose2d_matches_fp32(k, s, p, op):
    from flodl_b200 import ops
    torch.manual_seed(9)
    x = torch.randn(4, 16, 9, 11, device="cuda", requires_grad=True)
    w = torch.randn(16, 12, k, k, device="cuda", requires_grad=True)
    b = torch.randn(12, device="cuda", requires_grad=True)
    y = ops.conv_transpose2d(x, w, b, s, p, op)
    dy = torch.randn_like(y.float())
    y.float().backward(dy)
    x2, w2, b2 = [t.detach().clone().requires_grad_() for t in (x, w, b)]
    y2 = F.conv_transpose2d(x2.bfloat16().float(), w2.bfloat16().float(), b2, s, p, op)
    y2.backward(dy.bfloat16().float())
    assert y.shape == y2.shape
    for u, v in ((y.float(), y2), (x.grad, x2.grad), (w.grad, w2.grad), (b.grad, b2.grad)):
        assert ((u - v).norm() / v.norm()).item() < 1e-2


def test_conv_transpose1d_layer_matches_fp32():
    from flodl_b200.nn import ConvTranspose1d
    torch.manual_seed(10)
    m = ConvTranspose1d(8, 4, 4, stride=2, padding=1, device=torch.device("cuda"))
    x = torch.randn(6, 8, 50, device="cuda", requires_grad=True)
    y = m(x)
    dy = torch.randn_like(y.float())
    y.float().backward(dy)
    x2 = x.detach().clone().requires_grad_()
    w2 = m.weight.detach().clone().requires_grad_()
    b2 = m.bias.detach().clone().requires_grad_()
    y2 = F.conv_transpose1d(x2.bfloat16().float(), w2.bfloat16().float(), b2, 2, 1)
    y2.backward(dy.bfloat16().float())
    for u, v in ((y.float(), y2), (x.grad, x2.grad), (m.weight.grad, w2.grad),
                 (m.bias.grad, b2.grad)):
        assert ((u - v).norm() / v.norm()).item() < 1e-2


@pytest.mark.parametrize("M,N,K", [(4096, 16, 144), (8192, 64, 576), (2048, 40, 96)])
def test_gemm_column_sums_and_squares_feed_batch_norm(M, N, K):
    """The GEMM epilogue's per-column sum and sum of squares (kept per CTA in
    registers for a single N tile) and the batch norm applied from them match
    fp32 batch statistics of the same product; the workspace is left zeroed."""
    C_ = _C()
    torch.manual_seed(12)
    a = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ws = torch.zeros(2 * N + 1, device="cuda")
    C_.gemm(a, w, y, M, N, K, False, False, colsum=ws[:N], colsumsq=ws[N:2 * N])
    ref = a.float() @ w.float().t()
    torch.testing.assert_close(ws[:N], ref.sum(0), rtol=1e-3, atol=1e-2 * M ** 0.5)
    torch.testing.assert_close(ws[N:2 * N], (ref * ref).sum(0), rtol=1e-3, atol=1e-2 * M ** 0.5)
    mean = torch.empty(N, device="cuda")
    rstd = torch.empty(N, device="cuda")
    rm, rv = torch.zeros(N, device="cuda"), torch.ones(N, device="cuda")
    g, b = torch.rand(N, device="cuda") + 0.5, torch.randn(N, device="cuda")
    out = torch.empty_like(y)
    C_.bn_apply_sums(y, ws, mean, rstd, rm, rv, g, b, None, True, out, 1e-5, 0.1)
    torch.cuda.synchronize()
    mu, var = ref.mean(0), ref.var(0, unbiased=False)
    torch.testing.assert_close(mean, mu, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(rstd, (var + 1e-5).rsqrt(), rtol=2e-3, atol=1e-3)
    want = torch.relu((y.float() - mu) * (var + 1e-5).rsqrt() * g + b)
    torch.testing.assert_close(out.float(), want, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(rm, 0.1 * mu, rtol=1e-3, atol=1e-4)
    assert torch.count_nonzero(ws).item() == 0, "workspace not cleared for the next use"
