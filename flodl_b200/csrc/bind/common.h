// Shared helpers for the torch-facing bindings of the CUDA kernel library.
#pragma once
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#define FL_CHECK(cond, ...) TORCH_CHECK(cond, "flodl_b200: ", __VA_ARGS__)
#define FL_CHECK_CUDA(t) FL_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define FL_CHECK_BF16(t) FL_CHECK((t).scalar_type() == at::kBFloat16, #t " must be bf16")
#define FL_CHECK_F32(t) FL_CHECK((t).scalar_type() == at::kFloat, #t " must be f32")
// Error left in this thread's CUDA error slot by an earlier runtime call that
// is not ours (cudaGetLastError reports the last error of ANY call made by the
// thread). cur_stream() - evaluated by every binding right before it launches -
// moves it here, so the check after our launch reports our launch only.
inline const char*& stale_cuda_error() {
  thread_local const char* note = nullptr;
  return note;
}

#define FL_CUDA_OK(expr)                                                            \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    TORCH_CHECK(_e == cudaSuccess, "flodl_b200 CUDA error: ", cudaGetErrorString(_e), \
                " at ", __FILE__, ":", __LINE__,                                   \
                stale_cuda_error() ? " (an earlier call in this thread had left: " : "", \
                stale_cuda_error() ? stale_cuda_error() : "",                       \
                stale_cuda_error() ? ")" : "");                                     \
  } while (0)

inline cudaStream_t cur_stream() {
  cudaError_t e = cudaGetLastError();
  stale_cuda_error() = e == cudaSuccess ? nullptr : cudaGetErrorString(e);
  return at::cuda::getCurrentCUDAStream().stream();
}

template <typename T>
inline T* opt_ptr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

namespace py = pybind11;
void register_gemm(py::module& m);
void register_norm(py::module& m);
void register_attention(py::module& m);
void register_loss(py::module& m);
void register_optim(py::module& m);
void register_elementwise(py::module& m);
void register_conv(py::module& m);
void register_comm(py::module& m);
