"""Numerics of the tcgen05 GEMM engine against an fp32 PyTorch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from flodl_b200._ext import cuda_ext
    return cuda_ext()


def _ref(A, B, a_mn, b_mn):
    a = A.float().t() if a_mn else A.float()
    b = B.float().t() if b_mn else B.float()
    return a @ b.t()


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 512), (300, 200, 136), (1024, 1536, 512)])
def test_gemm_layouts(a_mn, b_mn, M, N, K):
    torch.manual_seed(0)
    C = _C()
    dev = "cuda"
    A = torch.randn((K, M) if a_mn else (M, K), device=dev).bfloat16()
    B = torch.randn((K, N) if b_mn else (N, K), device=dev).bfloat16()
    if a_mn and M % 8:
        pytest.skip("MN-major A needs M % 8 == 0")
    if b_mn and N % 8:
        pytest.skip("MN-major B needs N % 8 == 0")
    out = torch.empty(M, N, device=dev, dtype=torch.float32)
    C.gemm(A, B, out, M, N, K, a_mn, b_mn)
    torch.cuda.synchronize()
    ref = _ref(A, B, a_mn, b_mn)
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-3)


def test_gemm_bias_gelu_aux_bf16():
    torch.manual_seed(1)
    C = _C()
    M, N, K = 512, 768, 256
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.1).bfloat16()
    bias = torch.randn(N, device="cuda")
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    aux = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, B, out, M, N, K, False, False, bias=bias, aux=aux, flags=C.EPI_GELU)
    pre = (A.float() @ B.float().t() + bias).requires_grad_()
    g = torch.nn.functional.gelu(pre)
    g.backward(torch.ones_like(g))
    torch.testing.assert_close(out.float(), g.detach(), rtol=2e-2, atol=2e-2)
    # aux keeps GELU'(pre) for the backward pass
    torch.testing.assert_close(aux.float(), pre.grad, rtol=2e-2, atol=2e-2)


def test_gemm_residual_and_dgelu():
    torch.manual_seed(2)
    C = _C()
    M, N, K = 256, 512, 384
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.1).bfloat16()
    res = torch.randn(M, N, device="cuda")
    out = torch.empty(M, N, device="cuda")
    C.gemm(A, B, out, M, N, K, False, False, residual=res)
    torch.testing.assert_close(out, A.float() @ B.float().t() + res, rtol=1e-3, atol=1e-3)
    g = torch.rand(M, N, device="cuda").bfloat16()  # stored GELU' values
    out2 = torch.empty(M, N, device="cuda")
    C.gemm(A, B, out2, M, N, K, False, False, aux=g, flags=C.EPI_DGELU)
    torch.testing.assert_close(out2, (A.float() @ B.float().t()) * g.float(), rtol=1e-3, atol=1e-3)
    out3 = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)  # TMA epilogue path
    C.gemm(A, B, out3, M, N, K, False, False, aux=g, flags=C.EPI_DGELU)
    torch.testing.assert_close(out3.float(), (A.float() @ B.float().t()) * g.float(), rtol=2e-2,
                               atol=2e-2)


def test_gemm_splitk_accumulate():
    torch.manual_seed(3)
    C = _C()
    M, N, K = 512, 512, 8192
    A = torch.randn(K, M, device="cuda").bfloat16()  # dY stored [tokens, M]
    B = torch.randn(K, N, device="cuda").bfloat16()  # x stored [tokens, N]
    out = torch.ones(M, N, device="cuda")
    C.gemm(A, B, out, M, N, K, True, True, flags=C.EPI_ACCUMULATE, k_splits=8)
    ref = A.float().t() @ B.float() + 1.0
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=5e-2)


@pytest.mark.parametrize("M,N,K,b_mn", [(300, 512, 384, True), (16384 // 8, 2048, 512, True),
                                        (256, 200, 128, False)])
def test_gemm_fused_column_sums(M, N, K, b_mn):
    """colsum += column sums of the epilogue output (DGELU and plain), added to
    what the buffer already holds; partial row tiles contribute zeros."""
    torch.manual_seed(3)
    C = _C()
    A = torch.randn(M, K, device="cuda").bfloat16()
    Bm = (torch.randn(K, N, device="cuda") * 0.1).bfloat16() if b_mn else \
        (torch.randn(N, K, device="cuda") * 0.1).bfloat16()
    ref = _ref(A, Bm, False, b_mn)
    g = torch.rand(M, N, device="cuda").bfloat16()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cs = torch.full((N,), 0.5, device="cuda")
    C.gemm(A, Bm, out, M, N, K, False, b_mn, aux=g, flags=C.EPI_DGELU, colsum=cs)
    want = ref * g.float()
    torch.testing.assert_close(out.float(), want, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(cs, 0.5 + want.sum(0), rtol=1e-3, atol=1e-2 * (M ** 0.5))
    cs2 = torch.zeros(N, device="cuda")
    out2 = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, Bm, out2, M, N, K, False, b_mn, colsum=cs2)
    torch.testing.assert_close(cs2, ref.sum(0), rtol=1e-3, atol=1e-2 * (M ** 0.5))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(512, 512, 1024), (1000, 768, 2048), (2048, 1536, 1536)])
def test_cta_pair_tiles_match_fp32(M, N, K):
    """Long reductions (K >= 1024, M >= 512) run on CTA-pair tiles (one
    cta_group::2 MMA per 256-row tile): every operand layout and epilogue
    against a plain fp32 reference."""
    from flodl_b200._ext import cuda_ext
    C = cuda_ext()
    torch.manual_seed(1)
    bf = lambda *s: (torch.randn(*s, device="cuda") * 0.5).bfloat16()
    A, B, Bt, At = bf(M, K), bf(N, K), bf(K, N), bf(K, M)
    bias = torch.randn(N, device="cuda")

    def close(got, ref, tol=2e-2):
        err = (got.float() - ref).abs().max().item() / ref.abs().max().item()
        assert err < tol, err

    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, B, out, M, N, K, False, False, bias=bias)
    close(out, A.float() @ B.float().T + bias)
    C.gemm(A, Bt, out, M, N, K, False, True)
    close(out, A.float() @ Bt.float())
    res = torch.randn(M, N, device="cuda")
    o32 = torch.empty(M, N, device="cuda")
    C.gemm(A, B, o32, M, N, K, False, False, bias=bias, residual=res)
    close(o32, A.float() @ B.float().T + bias + res, 1e-3)
    aux = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, B, out, M, N, K, False, False, bias=bias, aux=aux, flags=C.EPI_GELU)
    close(out, torch.nn.functional.gelu(A.float() @ B.float().T + bias))
    g = torch.zeros(M, N, device="cuda")
    C.gemm(At, Bt, g, M, N, K, True, True, flags=C.EPI_ACCUMULATE)
    close(g, At.float().T @ Bt.float(), 1e-3)
    assert C.kernel_error() == 0


@pytest.mark.gpu
def test_192_column_tiles_match_fp32():
    """M = 4096, N = 1536 takes 192-column tiles (2 waves of 256 tiles of
    192 columns beat 2 waves of 192 tiles of 256 on 148 SMs): forward with
    bias, GELU, f32 residual, DGELU and an MN-major B against fp32."""
    from flodl_b200._ext import cuda_ext
    C = cuda_ext()
    torch.manual_seed(2)
    M, N, K = 4096, 1536, 512
    bf = lambda *s: (torch.randn(*s, device="cuda") * 0.5).bfloat16()
    A, B, Bt = bf(M, K), bf(N, K), bf(K, N)
    bias = torch.randn(N, device="cuda")

    def close(got, ref, tol=2e-2):
        err = (got.float() - ref).abs().max().item() / ref.abs().max().item()
        assert err < tol, err

    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, B, out, M, N, K, False, False, bias=bias)
    close(out, A.float() @ B.float().T + bias)
    aux = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, B, out, M, N, K, False, False, bias=bias, aux=aux, flags=C.EPI_GELU)
    close(out, torch.nn.functional.gelu(A.float() @ B.float().T + bias))
    res = torch.randn(M, N, device="cuda")
    o32 = torch.empty(M, N, device="cuda")
    C.gemm(A, B, o32, M, N, K, False, False, residual=res)
    close(o32, A.float() @ B.float().T + res, 1e-3)
    g = bf(M, N)
    C.gemm(A, Bt, out, M, N, K, False, True, aux=g, flags=C.EPI_DGELU)
    close(out, (A.float() @ Bt.float()) * g.float())
    assert C.kernel_error() == 0
