// Fused RMSNorm forward/backward for sm_100a (memory-bound, one warp per row).
//
// Reference: flodl/src/nn/rmsnorm.rs:54-62, which composes pow, mean, add,
// sqrt, div and mul (six passes over the row, each an allocation):
//   y = x * rstd * w,  rstd = 1 / sqrt(mean(x^2) + eps)
// Here one kernel reads x once per pass it needs (sum of squares, then the
// scaled write, the second pass hitting L1/L2) and keeps rstd per row for the
// backward:
//   g = dy * w,  xhat = x * rstd
//   dx = rstd * (g - xhat * mean(g * xhat))
//   dw += sum_rows dy * xhat   (per-lane register partials for rows up to 1024
//                               wide, else shared-memory atomics; one global
//                               atomic per column and block)
// x, y, dy and dx are f32 or bf16 (the same type); w, rstd and dw are f32.
#include "sm100_ptx.cuh"
#include "kernels.h"

namespace flodl {

namespace {

constexpr int kRmsThreads = 256;
constexpr int kRmsMaxC = 8192;  // the backward's shared-memory dw partials: 32 KB

__device__ __forceinline__ float ld_f32(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float ld_f32(const __nv_bfloat16* p, int64_t i) { return to_f32(p[i]); }
__device__ __forceinline__ void st_out(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void st_out(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kRmsThreads) rms_fwd_kernel(const T* __restrict__ x,
                                                              const float* __restrict__ w,
                                                              T* __restrict__ y,
                                                              float* __restrict__ rstd, int rows,
                                                              int C, float eps) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x / 32;
  for (int r = blockIdx.x * wpb + threadIdx.x / 32; r < rows; r += gridDim.x * wpb) {
    const T* xr = x + (int64_t)r * C;
    float ss = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float v = ld_f32(xr, c);
      ss = fmaf(v, v, ss);
    }
    const float rs = rsqrtf(warp_sum(ss) / (float)C + eps);
    T* yr = y + (int64_t)r * C;
    for (int c = lane; c < C; c += 32) st_out(yr, c, ld_f32(xr, c) * rs * (w ? __ldg(w + c) : 1.f));
    if (lane == 0 && rstd) rstd[r] = rs;
  }
}

// kRegDw: dw partials of a lane's columns (C <= 1024: at most 32) stay in
// registers across the warp's rows and meet in shared memory once per block;
// wider rows add into a shared-memory row with atomics.
template <typename T, bool kRegDw>
__global__ void __launch_bounds__(kRmsThreads) rms_bwd_kernel(
    const T* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ w,
    const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ dw, int rows, int C) {
  pdl_wait();
  pdl_trigger();
  constexpr int kWarps = kRmsThreads / 32;
  __shared__ float s_dw[kRegDw ? kWarps * 1024 : kRmsMaxC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
  float acc[32];
  if constexpr (kRegDw) {
#pragma unroll
    for (int k = 0; k < 32; ++k) acc[k] = 0.f;
  } else if (dw) {
    for (int c = threadIdx.x; c < C; c += blockDim.x) s_dw[c] = 0.f;
    __syncthreads();
  }
  for (int r = blockIdx.x * kWarps + warp; r < rows; r += gridDim.x * kWarps) {
    const T* xr = x + (int64_t)r * C;
    const T* gr = dy + (int64_t)r * C;
    const float rs = rstd[r];
    float dot = 0.f;  // sum of g * xhat
    if constexpr (kRegDw) {
      // the row stays in registers between the two passes
      float xv[32], gv[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const int c = lane + 32 * k;
        xv[k] = c < C ? ld_f32(xr, c) : 0.f;
        gv[k] = c < C ? ld_f32(gr, c) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const int c = lane + 32 * k;
        const float xh = xv[k] * rs;
        dot = fmaf(gv[k] * (c < C && w ? __ldg(w + c) : 1.f), xh, dot);
        acc[k] = fmaf(gv[k], xh, acc[k]);
      }
      const float m = warp_sum(dot) / (float)C;
      T* dr = dx + (int64_t)r * C;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const int c = lane + 32 * k;
        if (c < C) st_out(dr, c, rs * (gv[k] * (w ? __ldg(w + c) : 1.f) - xv[k] * rs * m));
      }
      continue;
    } else {
      for (int c = lane; c < C; c += 32) {
        const float xh = ld_f32(xr, c) * rs;
        const float d = ld_f32(gr, c);
        dot = fmaf(d * (w ? __ldg(w + c) : 1.f), xh, dot);
        if (dw) atomicAdd(&s_dw[c], d * xh);
      }
    }
    const float m = warp_sum(dot) / (float)C;
    T* dr = dx + (int64_t)r * C;
    for (int c = lane; c < C; c += 32) {
      const float xh = ld_f32(xr, c) * rs;
      const float g = ld_f32(gr, c) * (w ? __ldg(w + c) : 1.f);
      st_out(dr, c, rs * (g - xh * m));
    }
  }
  if (!dw) return;
  if constexpr (kRegDw) {
#pragma unroll
    for (int k = 0; k < 32; ++k)
      if (lane + 32 * k < C) s_dw[warp * 1024 + lane + 32 * k] = acc[k];
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int v = 0; v < kWarps; ++v) t += s_dw[v * 1024 + c];
      atomicAdd(dw + c, t);
    }
  } else {
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) atomicAdd(dw + c, s_dw[c]);
  }
}

int rms_grid(int rows, int per_sm) {
  const int wpb = kRmsThreads / 32;
  const int64_t b = ((int64_t)rows + wpb - 1) / wpb;
  const int64_t cap = (int64_t)num_sms() * per_sm;
  return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

}  // namespace

cudaError_t launch_rms_fwd(const void* x, bool bf16, const float* w, void* y, float* rstd,
                           int rows, int C, float eps, cudaStream_t st) {
  if (rows <= 0 || C <= 0) return cudaErrorInvalidValue;
  cudaError_t e;
  if (bf16)
    e = launch_pdl(rms_fwd_kernel<__nv_bfloat16>, dim3(rms_grid(rows, 8)), dim3(kRmsThreads), 0,
                   st, (const __nv_bfloat16*)x, w, (__nv_bfloat16*)y, rstd, rows, C, eps);
  else
    e = launch_pdl(rms_fwd_kernel<float>, dim3(rms_grid(rows, 8)), dim3(kRmsThreads), 0, st,
                   (const float*)x, w, (float*)y, rstd, rows, C, eps);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_rms_bwd(const void* dy, const void* x, bool bf16, const float* w,
                           const float* rstd, void* dx, float* dw, int rows, int C,
                           cudaStream_t st) {
  if (rows <= 0 || C <= 0 || (dw && C > kRmsMaxC)) return cudaErrorInvalidValue;
  const bool reg = C <= 1024;
  // with dw in shared-memory atomics, fewer blocks (one flush each)
  const int grid = rms_grid(rows, (dw && !reg) ? 2 : 8);
  cudaError_t e;
  if (bf16) {
    auto k = reg ? rms_bwd_kernel<__nv_bfloat16, true> : rms_bwd_kernel<__nv_bfloat16, false>;
    e = launch_pdl(k, dim3(grid), dim3(kRmsThreads), 0, st, (const __nv_bfloat16*)dy,
                   (const __nv_bfloat16*)x, w, rstd, (__nv_bfloat16*)dx, dw, rows, C);
  } else {
    auto k = reg ? rms_bwd_kernel<float, true> : rms_bwd_kernel<float, false>;
    e = launch_pdl(k, dim3(grid), dim3(kRmsThreads), 0, st, (const float*)dy, (const float*)x, w,
                   rstd, (float*)dx, dw, rows, C);
  }
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
