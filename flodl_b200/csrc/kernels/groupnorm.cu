// Fused GroupNorm forward/backward for sm_100a (memory-bound, one CTA per
// (sample, group) row).
//
// Reference: flodl/src/nn/groupnorm.rs:62-70 (libtorch group_norm through the shim).
// x is [N, C, *] contiguous, so the Cg = C / G channels of group g of sample n
// are one contiguous row of L = Cg * HW elements:
//   y = (x - mean) * rstd * gamma[c] + beta[c],  rstd = 1 / sqrt(var + eps)
// (biased variance over the row, two passes for its accuracy). Backward, with
// xhat = (x - mean) * rstd and g = dy * gamma[c]:
//   dx = rstd * (g - mean(g) - xhat * mean(g * xhat))
//   dgamma[c] += sum dy * xhat,  dbeta[c] += sum dy   (over the HW elements of
//                                                      channel c, all samples)
// Warps take whole channels (HW contiguous elements), so the per-channel sums
// need one warp reduction and one atomic each. x/y/dy/dx are f32 or bf16.
#include "sm100_ptx.cuh"
#include "kernels.h"

namespace flodl {

namespace {

constexpr int kGnThreads = 256;
constexpr int kGnWarps = kGnThreads / 32;

__device__ __forceinline__ float gn_ld(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float gn_ld(const __nv_bfloat16* p, int64_t i) { return to_f32(p[i]); }
__device__ __forceinline__ void gn_st(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void gn_st(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float gn_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum of v over the CTA (every thread gets it).
__device__ __forceinline__ float gn_block_sum(float v, float* red) {
  v = gn_warp_sum(v);
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read from a previous call
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kGnWarps; ++i) s += red[i];
  return s;
}

template <typename T>
__global__ void __launch_bounds__(kGnThreads) gn_fwd_kernel(
    const T* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    T* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out, int rows, int G,
    int Cg, int HW, float eps) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[kGnWarps];
  const int64_t L = (int64_t)Cg * HW;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + (int64_t)r * L;
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < L; i += blockDim.x) s += gn_ld(xr, i);
    const float mean = gn_block_sum(s, red) / (float)L;
    float q = 0.f;
    for (int64_t i = threadIdx.x; i < L; i += blockDim.x) {
      const float d = gn_ld(xr, i) - mean;
      q = fmaf(d, d, q);
    }
    const float rstd = rsqrtf(gn_block_sum(q, red) / (float)L + eps);
    const int c0 = (r % G) * Cg;
    T* yr = y + (int64_t)r * L;
    const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
    for (int cl = w; cl < Cg; cl += kGnWarps) {
      const float ga = gamma ? __ldg(gamma + c0 + cl) : 1.f;
      const float be = beta ? __ldg(beta + c0 + cl) : 0.f;
      const float a = rstd * ga, b = be - mean * rstd * ga;
      const int64_t base = (int64_t)cl * HW;
      for (int i = lane; i < HW; i += 32) gn_st(yr, base + i, fmaf(gn_ld(xr, base + i), a, b));
    }
    if (threadIdx.x == 0) {
      mean_out[r] = mean;
      rstd_out[r] = rstd;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kGnThreads) gn_bwd_kernel(
    const T* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ gamma,
    const float* __restrict__ mean_in, const float* __restrict__ rstd_in, T* __restrict__ dx,
    float* __restrict__ dgamma, float* __restrict__ dbeta, int rows, int G, int Cg, int HW) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[kGnWarps];
  const int64_t L = (int64_t)Cg * HW;
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + (int64_t)r * L;
    const T* gr = dy + (int64_t)r * L;
    const float mean = mean_in[r], rstd = rstd_in[r];
    const int c0 = (r % G) * Cg;
    // per channel: sum dy and sum dy * xhat; the row's sums of g and g * xhat
    float a = 0.f, b = 0.f;
    for (int cl = w; cl < Cg; cl += kGnWarps) {
      const int64_t base = (int64_t)cl * HW;
      float sd = 0.f, sdx = 0.f;
      for (int i = lane; i < HW; i += 32) {
        const float d = gn_ld(gr, base + i);
        sd += d;
        sdx = fmaf(d, (gn_ld(xr, base + i) - mean) * rstd, sdx);
      }
      sd = gn_warp_sum(sd);
      sdx = gn_warp_sum(sdx);
      const float ga = gamma ? __ldg(gamma + c0 + cl) : 1.f;
      a = fmaf(ga, sd, a);
      b = fmaf(ga, sdx, b);
      if (lane == 0) {
        if (dbeta) atomicAdd(dbeta + c0 + cl, sd);
        if (dgamma) atomicAdd(dgamma + c0 + cl, sdx);
      }
    }
    // a, b are warp-uniform: one lane per warp contributes
    const float ma = gn_block_sum(lane == 0 ? a : 0.f, red) / (float)L;
    const float mb = gn_block_sum(lane == 0 ? b : 0.f, red) / (float)L;
    T* dr = dx + (int64_t)r * L;
    for (int cl = w; cl < Cg; cl += kGnWarps) {
      const float ga = gamma ? __ldg(gamma + c0 + cl) : 1.f;
      const int64_t base = (int64_t)cl * HW;
      for (int i = lane; i < HW; i += 32) {
        const float xh = (gn_ld(xr, base + i) - mean) * rstd;
        gn_st(dr, base + i, rstd * (gn_ld(gr, base + i) * ga - ma - xh * mb));
      }
    }
  }
}

int gn_grid(int rows) {
  const int cap = num_sms() * 8;
  return rows < cap ? (rows > 0 ? rows : 1) : cap;
}

}  // namespace

cudaError_t launch_gn_fwd(const void* x, bool bf16, const float* gamma, const float* beta,
                          void* y, float* mean, float* rstd, int N, int C, int HW, int G,
                          float eps, cudaStream_t st) {
  if (N <= 0 || C <= 0 || HW <= 0 || G <= 0 || C % G) return cudaErrorInvalidValue;
  const int rows = N * G, Cg = C / G;
  cudaError_t e;
  if (bf16)
    e = launch_pdl(gn_fwd_kernel<__nv_bfloat16>, dim3(gn_grid(rows)), dim3(kGnThreads), 0, st,
                   (const __nv_bfloat16*)x, gamma, beta, (__nv_bfloat16*)y, mean, rstd, rows, G,
                   Cg, HW, eps);
  else
    e = launch_pdl(gn_fwd_kernel<float>, dim3(gn_grid(rows)), dim3(kGnThreads), 0, st,
                   (const float*)x, gamma, beta, (float*)y, mean, rstd, rows, G, Cg, HW, eps);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_gn_bwd(const void* dy, const void* x, bool bf16, const float* gamma,
                          const float* mean, const float* rstd, void* dx, float* dgamma,
                          float* dbeta, int N, int C, int HW, int G, cudaStream_t st) {
  if (N <= 0 || C <= 0 || HW <= 0 || G <= 0 || C % G) return cudaErrorInvalidValue;
  const int rows = N * G, Cg = C / G;
  cudaError_t e;
  if (bf16)
    e = launch_pdl(gn_bwd_kernel<__nv_bfloat16>, dim3(gn_grid(rows)), dim3(kGnThreads), 0, st,
                   (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, gamma, mean, rstd,
                   (__nv_bfloat16*)dx, dgamma, dbeta, rows, G, Cg, HW);
  else
    e = launch_pdl(gn_bwd_kernel<float>, dim3(gn_grid(rows)), dim3(kGnThreads), 0, st,
                   (const float*)dy, (const float*)x, gamma, mean, rstd, (float*)dx, dgamma,
                   dbeta, rows, G, Cg, HW);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
