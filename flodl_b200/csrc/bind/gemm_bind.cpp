// Torch bindings for the tcgen05 GEMM engine.
#include "common.h"
#include "../kernels/gemm_sm100.h"

namespace {

// out = epilogue(op(A) @ op(B)^T). Shapes are given by the caller (the Python
// op layer); this function validates pointers, dtypes and alignment.
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t M, int64_t N,
          int64_t K, bool a_mn, bool b_mn, const c10::optional<at::Tensor>& bias,
          const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& aux,
          int64_t flags, double alpha, int64_t k_splits, int64_t bn,
          const c10::optional<at::Tensor>& alpha_t, const c10::optional<at::Tensor>& colsum,
          const c10::optional<at::Tensor>& colsumsq) {
  FL_CHECK_CUDA(A);
  FL_CHECK_CUDA(B);
  FL_CHECK_CUDA(out);
  FL_CHECK_BF16(A);
  FL_CHECK_BF16(B);
  FL_CHECK(A.dim() == 2 && B.dim() == 2 && out.dim() == 2, "gemm operands must be 2-D");
  FL_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && out.stride(1) == 1,
           "gemm operands must be row-major");
  // A stored [M,K] (or [K,M] when a_mn); B stored [N,K] (or [K,N] when b_mn).
  FL_CHECK(a_mn ? (A.size(0) == K && A.size(1) == M) : (A.size(0) == M && A.size(1) == K),
           "A shape mismatch");
  FL_CHECK(b_mn ? (B.size(0) == K && B.size(1) == N) : (B.size(0) == N && B.size(1) == K),
           "B shape mismatch");
  FL_CHECK(out.size(0) == M && out.size(1) == N, "out shape mismatch");
  FL_CHECK(A.stride(0) % 8 == 0 && B.stride(0) % 8 == 0, "row pitch must be a multiple of 16 bytes");
  FL_CHECK(reinterpret_cast<uintptr_t>(A.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(B.data_ptr()) % 16 == 0,
           "operands must be 16-byte aligned");
  const bool out_f32 = out.scalar_type() == at::kFloat;
  FL_CHECK(out_f32 || out.scalar_type() == at::kBFloat16, "out must be bf16 or f32");
  if (k_splits > 1) FL_CHECK(out_f32 && (flags & flodl::kEpiAccumulate), "split-K needs f32 accumulate");
  if (flags & flodl::kEpiAccumulate) FL_CHECK(out_f32, "accumulate needs f32 out");
  if (bias) { FL_CHECK_F32(*bias); FL_CHECK(bias->numel() == N && bias->is_contiguous(), "bias"); }
  if (residual) {
    FL_CHECK_F32(*residual);
    FL_CHECK(residual->dim() == 2 && residual->size(0) == M && residual->size(1) == N &&
                 residual->stride(1) == 1, "residual shape");
  }
  if (flags & (flodl::kEpiDGelu)) FL_CHECK(aux.has_value(), "dgelu needs aux");
  if (aux) {
    FL_CHECK_BF16(*aux);
    FL_CHECK(aux->dim() == 2 && aux->size(0) == M && aux->size(1) == N && aux->stride(1) == 1,
             "aux shape");
  }
  c10::cuda::CUDAGuard guard(A.device());
  flodl::GemmArgs g;
  g.A = A.data_ptr();
  g.B = B.data_ptr();
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.lda = (int)A.stride(0);
  g.ldb = (int)B.stride(0);
  g.a_mn = a_mn;
  g.b_mn = b_mn;
  g.k_splits = (int)k_splits;
  g.bn = (int)bn;
  g.ep.out = out.data_ptr();
  g.ep.ld_out = (int)out.stride(0);
  g.ep.out_f32 = out_f32 ? 1 : 0;
  g.ep.bias = opt_ptr<const float>(bias);
  g.ep.residual = opt_ptr<const float>(residual);
  g.ep.ld_res = residual ? (int)residual->stride(0) : 0;
  g.ep.aux = opt_ptr<void>(aux);
  g.ep.ld_aux = aux ? (int)aux->stride(0) : 0;
  g.ep.flags = (int)flags;
  g.ep.alpha = (float)alpha;
  if (alpha_t) { FL_CHECK_F32(*alpha_t); FL_CHECK_CUDA(*alpha_t); }
  g.ep.alpha_ptr = opt_ptr<const float>(alpha_t);
  if (colsum) {
    FL_CHECK_F32(*colsum);
    FL_CHECK_CUDA(*colsum);
    FL_CHECK(colsum->numel() == N && colsum->is_contiguous(), "colsum must be f32 [N]");
    FL_CHECK(k_splits == 1 && !(flags & flodl::kEpiAccumulate), "colsum needs a full-K epilogue");
  }
  g.ep.colsum = opt_ptr<float>(colsum);
  if (colsumsq) {
    FL_CHECK_F32(*colsumsq);
    FL_CHECK_CUDA(*colsumsq);
    FL_CHECK(colsumsq->numel() == N && colsumsq->is_contiguous(), "colsumsq must be f32 [N]");
    FL_CHECK(k_splits == 1 && !(flags & flodl::kEpiAccumulate),
             "colsumsq needs a full-K epilogue");
  }
  g.ep.colsumsq = opt_ptr<float>(colsumsq);
  cudaStream_t st = cur_stream();
  cudaError_t e = flodl::launch_gemm(g, st);
  FL_CHECK(e == cudaSuccess, "gemm launch failed: ", cudaGetErrorString(e), " ",
           flodl::gemm_failure_detail(), " [M=", M, " N=", N, " K=", K, " a_mn=", a_mn,
           " b_mn=", b_mn, " splits=", k_splits, "]",
           stale_cuda_error() ? " (an earlier call in this thread had left: " : "",
           stale_cuda_error() ? stale_cuda_error() : "", stale_cuda_error() ? ")" : "");
}

}  // namespace

void register_gemm(py::module& m) {
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM with fused epilogue", py::arg("A"), py::arg("B"),
        py::arg("out"), py::arg("M"), py::arg("N"), py::arg("K"), py::arg("a_mn"),
        py::arg("b_mn"), py::arg("bias") = py::none(), py::arg("residual") = py::none(),
        py::arg("aux") = py::none(), py::arg("flags") = 0, py::arg("alpha") = 1.0,
        py::arg("k_splits") = 1, py::arg("bn") = 0, py::arg("alpha_t") = py::none(),
        py::arg("colsum") = py::none(), py::arg("colsumsq") = py::none());
  m.attr("EPI_GELU") = (int)flodl::kEpiGelu;
  m.attr("EPI_DGELU") = (int)flodl::kEpiDGelu;
  m.attr("EPI_ACCUMULATE") = (int)flodl::kEpiAccumulate;
  m.def("num_sms", &flodl::num_sms);
  m.def("launch_count", &flodl::launch_count, "kernels launched by this library so far");
  m.def("reset_launch_count", &flodl::reset_launch_count);
  m.def("kernel_error", &flodl::read_kernel_error,
        "nonzero if a bounded wait in a compute kernel expired (1 = mbarrier timeout)");
  m.def("clear_kernel_error", &flodl::clear_kernel_error);
  m.def("set_wait_limit_ns", [](int64_t ns) { flodl::set_wait_limit_ns((uint64_t)ns); });
}
