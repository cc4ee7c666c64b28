// Dropout for sm_100a with a counter-based generator, so that the backward
// regenerates the mask instead of storing it (reference: at::dropout through
// flodl-sys/ops_nn.cpp; flodl/src/nn/dropout.rs).
//
// Random bits: Philox-4x32 with 10 rounds (Salmon, Moraes, Dror and Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011): counter =
// (element group lo, hi, call offset lo, hi), key = (seed lo, hi); each
// call gives four 32-bit words, one per element of a group of four. Element i
// is kept when its word >= p * 2^32, and a kept element is scaled by 1/(1-p).
// x/y/dy/dx are f32 or bf16.
#include "sm100_ptx.cuh"
#include "kernels.h"

namespace flodl {

namespace {

// Philox-4x32 constants from the paper (round multipliers and Weyl key
// increments).
constexpr uint32_t kPhiloxM0 = 0xD2511F53u, kPhiloxM1 = 0xCD9E8D57u;
constexpr uint32_t kPhiloxW0 = 0x9E3779B9u, kPhiloxW1 = 0xBB67AE85u;

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kPhiloxM0, c.x), lo0 = kPhiloxM0 * c.x;
    const uint32_t hi1 = __umulhi(kPhiloxM1, c.z), lo1 = kPhiloxM1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += kPhiloxW0;
    k.y += kPhiloxW1;
  }
  return c;
}

__device__ __forceinline__ float dr_ld(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float dr_ld(const __nv_bfloat16* p, int64_t i) { return to_f32(p[i]); }
__device__ __forceinline__ void dr_st(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void dr_st(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

// y = x * keep / (1 - p) for the forward; the backward applies the same
// mask to dy (the same seed and offset regenerate it).
template <typename T>
__global__ void dropout_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n,
                               uint32_t threshold, float scale, uint64_t seed, uint64_t offset) {
  pdl_wait();
  pdl_trigger();
  const int64_t groups = (n + 3) / 4;
  const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    const uint4 r = philox4x32_10(make_uint4((uint32_t)g, (uint32_t)((uint64_t)g >> 32),
                                             (uint32_t)offset, (uint32_t)(offset >> 32)),
                                  key);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int64_t i = g * 4 + e;
      if (i < n) dr_st(y, i, w[e] >= threshold ? dr_ld(x, i) * scale : 0.f);
    }
  }
}

}  // namespace

cudaError_t launch_dropout(const void* x, void* y, bool bf16, int64_t n, float p, uint64_t seed,
                           uint64_t offset, cudaStream_t st) {
  if (n <= 0 || !(p >= 0.f) || !(p < 1.f)) return cudaErrorInvalidValue;
  const double t = (double)p * 4294967296.0;  // keep when the word is >= p * 2^32
  const uint32_t threshold = t >= 4294967295.0 ? 0xffffffffu : (uint32_t)t;
  const float scale = 1.f / (1.f - p);
  const int64_t groups = (n + 3) / 4;
  const int64_t b = (groups + 255) / 256, cap = (int64_t)num_sms() * 16;
  const int grid = (int)(b < cap ? (b > 0 ? b : 1) : cap);
  cudaError_t e;
  if (bf16)
    e = launch_pdl(dropout_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st,
                   (const __nv_bfloat16*)x, (__nv_bfloat16*)y, n, threshold, scale, seed, offset);
  else
    e = launch_pdl(dropout_kernel<float>, dim3(grid), dim3(256), 0, st, (const float*)x, (float*)y,
                   n, threshold, scale, seed, offset);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
