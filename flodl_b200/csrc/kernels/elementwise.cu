// Standalone elementwise kernels used where no producing GEMM can absorb the
// operation in its epilogue (e.g. a GELU module between two non-fused layers).
#include "sm100_ptx.cuh"
#include "kernels.h"

namespace flodl {

namespace {

int grid_1d(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * 8;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

__global__ void gelu_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                const __nv_bfloat16* __restrict__ h, __nv_bfloat16* __restrict__ dh,
                                int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    dh[i] = __float2bfloat16_rn(__bfloat162float(dy[i]) * gelu_erf_grad(__bfloat162float(h[i])));
}

__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = __float2bfloat16_rn(gelu_erf(__bfloat162float(x[i])));
}

// f32 GELU and GELU' exactly as the GEMM epilogues evaluate them (numerics tests).
__global__ void gelu_eval_f32_kernel(const float* __restrict__ x, float* __restrict__ y,
                                     float* __restrict__ dydx, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    y[i] = gelu_erf(x[i]);
    dydx[i] = gelu_erf_grad(x[i]);
  }
}

__global__ void mul_bf16_kernel(const __nv_bfloat16* __restrict__ a,
                                const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ y,
                                int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = __float2bfloat16_rn(__bfloat162float(a[i]) * __bfloat162float(b[i]));
}

}  // namespace

cudaError_t launch_mul_bf16(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* y,
                            int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  mul_bf16_kernel<<<grid_1d(n, 256), 256, 0, st>>>(a, b, y, n);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_gelu_eval_f32(const float* x, float* y, float* dydx, int64_t n,
                                 cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  gelu_eval_f32_kernel<<<grid_1d(n, 256), 256, 0, st>>>(x, y, dydx, n);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_gelu_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* h, __nv_bfloat16* dh,
                            int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  gelu_bwd_kernel<<<grid_1d(n, 256), 256, 0, st>>>(dy, h, dh, n);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_gelu_fwd(const __nv_bfloat16* x, __nv_bfloat16* y, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  gelu_fwd_kernel<<<grid_1d(n, 256), 256, 0, st>>>(x, y, n);
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
