"""The C interface of the kernel library (flodl_b200/csrc/capi/flodl.h).

CPU: the header compiles as C99 and as C++17 on its own; every function it
declares is exported by the built extension; argument checks answer before
any CUDA call with a negative status and a message from flodl_last_error().
GPU: the C entry points, called through ctypes with raw device pointers,
match plain PyTorch fp32 references of the same ops.

Reference seam: flodl-sys/shim.h (the reference's `extern "C"` functions with
error strings, bound by its Rust crate).
"""
import ctypes
import os
import re
import shutil
import subprocess

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "flodl_b200", "csrc", "capi", "flodl.h")


def _lib():
    from flodl_b200._ext import cuda_ext
    mod = cuda_ext()
    return ctypes.CDLL(mod.__file__)


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(flodl_[a-z0-9_]+)\s*\(", text)))


@pytest.mark.parametrize("lang,std", [("c", "-std=c99"), ("c++", "-std=c++17")])
def test_header_compiles_standalone(tmp_path, lang, std):
    cc = shutil.which("gcc" if lang == "c" else "g++")
    if cc is None:
        pytest.skip("no host compiler")
    src = tmp_path / ("t.c" if lang == "c" else "t.cpp")
    src.write_text('#include "flodl.h"\nint main(void) { flodl_gemm_desc d; (void)d; '
                   'return FLODL_OK; }\n')
    r = subprocess.run([cc, std, "-Wall", "-Wextra", "-Werror", "-fsyntax-only",
                        "-I", os.path.dirname(HEADER), str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_every_declared_function_is_exported():
    lib = _lib()
    names = _declared()
    assert len(names) >= 24
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_argument_errors_answer_before_cuda():
    lib = _lib()
    lib.flodl_last_error.restype = ctypes.c_char_p
    assert lib.flodl_abi_version() == 1
    # a NULL descriptor
    assert lib.flodl_gemm_bf16(None, None) == -1
    assert b"desc is NULL" in lib.flodl_last_error()
    # a LayerNorm width the kernels do not cover: unsupported, not a crash
    fake = ctypes.c_void_p(16)
    rc = lib.flodl_layer_norm_fwd(fake, 0, None, None, fake, None, fake, fake, 4, 6,
                                  ctypes.c_float(1e-5), None)
    assert rc == -2 and b"multiple of 4" in lib.flodl_last_error()
    rc = lib.flodl_flash_attn_fwd(fake, fake, fake, None, 1, 128, 1, 32, 1,
                                  ctypes.c_float(0.125), None)
    assert rc == -2 and b"head_dim" in lib.flodl_last_error()
    rc = lib.flodl_sgd_step(fake, fake, None, None, ctypes.c_int64(8), fake, None, None,
                            ctypes.c_float(0.9), ctypes.c_float(0.0), ctypes.c_float(0.0), 0, 0,
                            None)
    assert rc == -1 and b"momentum needs buf" in lib.flodl_last_error()


# ------------------------------------------------------------------ GPU
def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class GemmDesc(ctypes.Structure):
    _fields_ = [("A", ctypes.c_void_p), ("B", ctypes.c_void_p), ("M", ctypes.c_int),
                ("N", ctypes.c_int), ("K", ctypes.c_int), ("lda", ctypes.c_int),
                ("ldb", ctypes.c_int), ("a_trans", ctypes.c_int), ("b_trans", ctypes.c_int),
                ("out", ctypes.c_void_p), ("ld_out", ctypes.c_int), ("out_f32", ctypes.c_int),
                ("bias", ctypes.c_void_p), ("residual", ctypes.c_void_p),
                ("ld_res", ctypes.c_int), ("aux", ctypes.c_void_p), ("ld_aux", ctypes.c_int),
                ("flags", ctypes.c_int), ("alpha", ctypes.c_float), ("k_splits", ctypes.c_int)]


@pytest.mark.gpu
def test_gemm_bias_gelu_through_c_matches_fp32():
    lib = _lib()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    M, N, K = 1024, 768, 512
    a = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(N, K, device=dev) / K ** 0.5).bfloat16()
    bias = torch.randn(N, device=dev)
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    aux = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    d = GemmDesc(A=a.data_ptr(), B=w.data_ptr(), M=M, N=N, K=K, lda=K, ldb=K, a_trans=0,
                 b_trans=0, out=out.data_ptr(), ld_out=N, out_f32=0, bias=bias.data_ptr(),
                 residual=None, ld_res=0, aux=aux.data_ptr(), ld_aux=N, flags=1, alpha=1.0,
                 k_splits=1)
    assert lib.flodl_gemm_bf16(ctypes.byref(d), _stream()) == 0
    torch.cuda.synchronize()
    pre = a.float() @ w.float().t() + bias
    want = torch.nn.functional.gelu(pre)
    assert torch.allclose(out.float(), want, atol=3e-2, rtol=2e-2)
    assert lib.flodl_kernel_error() == 0


@pytest.mark.gpu
def test_layer_norm_and_adamw_through_c_match_fp32():
    lib = _lib()
    dev = torch.device("cuda", 0)
    torch.manual_seed(1)
    rows, C = 4096, 512
    x = torch.randn(rows, C, device=dev)
    g = torch.randn(C, device=dev)
    b = torch.randn(C, device=dev)
    y = torch.empty(rows, C, device=dev)
    mean = torch.empty(rows, device=dev)
    rstd = torch.empty(rows, device=dev)
    rc = lib.flodl_layer_norm_fwd(_p(x), 0, _p(g), _p(b), None, _p(y), _p(mean), _p(rstd), rows,
                                  C, ctypes.c_float(1e-5), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    want = torch.nn.functional.layer_norm(x, (C,), g, b, 1e-5)
    assert torch.allclose(y, want, atol=1e-4, rtol=1e-4)

    n = 1 << 20
    p = torch.randn(n, device=dev)
    grad = torch.randn(n, device=dev)
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    lr = torch.tensor([1e-3], device=dev)
    step = torch.tensor([1.0], device=dev)
    ref = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.1)
    ref.grad = grad.clone()
    opt.step()
    rc = lib.flodl_adamw_step(_p(p), _p(grad), _p(m), _p(v), None, ctypes.c_int64(n), _p(lr),
                              _p(step), None, ctypes.c_float(0.9), ctypes.c_float(0.999),
                              ctypes.c_float(1e-8), ctypes.c_float(0.1), 1, 0, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.allclose(p, ref.detach(), atol=1e-6, rtol=1e-5)


@pytest.mark.gpu
def test_flash_attention_and_cross_entropy_through_c_match_fp32():
    lib = _lib()
    dev = torch.device("cuda", 0)
    torch.manual_seed(2)
    B, S, H, D = 2, 256, 4, 64
    qkv = torch.randn(B * S, 3 * H * D, device=dev).bfloat16()
    out = torch.empty(B * S, H * D, device=dev, dtype=torch.bfloat16)
    lse2 = torch.empty(B, H, S, device=dev)
    rc = lib.flodl_flash_attn_fwd(_p(qkv), _p(out), _p(lse2), None, B, S, H, D, 1,
                                  ctypes.c_float(D ** -0.5), _stream())
    assert rc == 0, ctypes.string_at(lib.flodl_last_error())
    torch.cuda.synchronize()
    q, k, v = qkv.float().view(B, S, 3, H, D).permute(2, 0, 3, 1, 4)
    want = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    want = want.permute(0, 2, 1, 3).reshape(B * S, H * D)
    assert (out.float() - want).abs().max().item() < 2e-2

    T, V = 1000, 256
    logits = torch.randn(T, V, device=dev).bfloat16()
    tgt = torch.randint(0, V, (T,), device=dev)
    tgt[::7] = -100
    loss = torch.zeros(1, device=dev)
    inv = torch.zeros(1, device=dev)
    dl = torch.empty(T, V, device=dev, dtype=torch.bfloat16)
    rc = lib.flodl_softmax_cross_entropy(_p(logits), V, _p(tgt), T, V, ctypes.c_int64(-100),
                                         ctypes.c_float(0.0), _p(loss), _p(dl), _p(inv),
                                         _stream())
    assert rc == 0
    torch.cuda.synchronize()
    lf = logits.float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(lf, tgt, ignore_index=-100)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 1e-3
    assert torch.allclose(dl.float(), lf.grad, atol=1e-4)
