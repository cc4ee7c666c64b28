// Max pooling over NCHW planes for sm_100a (reference: at::max_pool2d through
// flodl-sys/ops_nn.cpp; flodl/src/nn/pooling.rs). Forward keeps the flat
// in-plane index of each window's maximum (int32), so the backward is a
// scatter of dy to those positions (atomic adds: windows overlap when the
// stride is below the kernel extent). A window's maximum is its first
// largest element in row-major order; NaN inputs win (they propagate, as in
// PyTorch). x/y/dy/dx are f32 or bf16; dx must start zeroed.
#include "sm100_ptx.cuh"
#include "kernels.h"

namespace flodl {

namespace {

__device__ __forceinline__ float mp_ld(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float mp_ld(const __nv_bfloat16* p, int64_t i) { return to_f32(p[i]); }
__device__ __forceinline__ void mp_st(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void mp_st(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}
__device__ __forceinline__ void mp_add(float* p, float v) { atomicAdd(p, v); }
__device__ __forceinline__ void mp_add(__nv_bfloat16* p, float v) {
  atomicAdd(p, __float2bfloat16_rn(v));
}

template <typename T>
__global__ void maxpool_fwd_kernel(const T* __restrict__ x, T* __restrict__ y,
                                   int32_t* __restrict__ idx, int planes, int H, int W, int Ho,
                                   int Wo, PoolGeo g, FastDiv fWo, FastDiv fHo) {
  pdl_wait();
  pdl_trigger();
  const uint32_t total = (uint32_t)planes * Ho * Wo;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t t = fWo.div(i);
    const int ow = (int)(i - t * Wo);
    const uint32_t pl = fHo.div(t);
    const int oh = (int)(t - pl * Ho);
    const T* xp = x + (int64_t)pl * H * W;
    const int h0 = oh * g.sh - g.ph, w0 = ow * g.sw - g.pw;
    float best = -INFINITY;
    int bi = -1;
    for (int kh = 0; kh < g.kh; ++kh) {
      const int h = h0 + kh * g.dh;
      if (h < 0 || h >= H) continue;
      for (int kw = 0; kw < g.kw; ++kw) {
        const int w = w0 + kw * g.dw;
        if (w < 0 || w >= W) continue;
        const float v = mp_ld(xp, (int64_t)h * W + w);
        if (v > best || v != v || bi < 0) {
          if (!(best != best)) {  // keep the first NaN
            best = v;
            bi = h * W + w;
          }
        }
      }
    }
    mp_st(y, i, best);
    idx[i] = bi;
  }
}

// The common 2x2 window, stride 2, no padding or dilation, every window
// inside the input: four loads per output and no bounds checks.
template <typename T>
__global__ void maxpool2x2_fwd_kernel(const T* __restrict__ x, T* __restrict__ y,
                                      int32_t* __restrict__ idx, int planes, int H, int W, int Ho,
                                      int Wo, FastDiv fWo, FastDiv fHo) {
  pdl_wait();
  pdl_trigger();
  const uint32_t total = (uint32_t)planes * Ho * Wo;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t t = fWo.div(i);
    const int ow = (int)(i - t * Wo);
    const uint32_t pl = fHo.div(t);
    const int oh = (int)(t - pl * Ho);
    const int j0 = 2 * oh * W + 2 * ow;
    const T* xp = x + (int64_t)pl * H * W;
    const int js[4] = {j0, j0 + 1, j0 + W, j0 + W + 1};
    float best = mp_ld(xp, js[0]);
    int bi = js[0];
#pragma unroll
    for (int q = 1; q < 4; ++q) {
      const float v = mp_ld(xp, js[q]);
      if ((v > best || v != v) && !(best != best)) {  // first maximum; the first NaN wins
        best = v;
        bi = js[q];
      }
    }
    mp_st(y, i, best);
    idx[i] = bi;
  }
}

template <typename T>
__global__ void maxpool_bwd_kernel(const T* __restrict__ dy, const int32_t* __restrict__ idx,
                                   T* __restrict__ dx, int planes, int HW, int HoWo,
                                   FastDiv fHoWo) {
  pdl_wait();
  pdl_trigger();
  const uint32_t total = (uint32_t)planes * HoWo;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int j = idx[i];
    if (j < 0) continue;
    const uint32_t pl = fHoWo.div(i);
    mp_add(dx + (int64_t)pl * HW + j, mp_ld(dy, i));
  }
}

int pool_grid(int64_t work) {
  const int64_t b = (work + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 16;
  return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

}  // namespace

cudaError_t launch_maxpool_fwd(const void* x, bool bf16, void* y, int32_t* idx, int planes, int H,
                               int W, int Ho, int Wo, const PoolGeo& g, cudaStream_t st) {
  if (planes <= 0 || Ho <= 0 || Wo <= 0 || g.kh <= 0 || g.kw <= 0 || g.sh <= 0 || g.sw <= 0 ||
      g.dh <= 0 || g.dw <= 0 || (int64_t)planes * Ho * Wo >= kMaxFlatIndex ||
      (int64_t)H * W >= kMaxFlatIndex)
    return cudaErrorInvalidValue;
  const int grid = pool_grid((int64_t)planes * Ho * Wo);
  const bool k2s2 = g.kh == 2 && g.kw == 2 && g.sh == 2 && g.sw == 2 && g.ph == 0 && g.pw == 0 &&
                    g.dh == 1 && g.dw == 1 && 2 * Ho <= H && 2 * Wo <= W;
  cudaError_t e;
  if (k2s2 && bf16)
    e = launch_pdl(maxpool2x2_fwd_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st,
                   (const __nv_bfloat16*)x, (__nv_bfloat16*)y, idx, planes, H, W, Ho, Wo,
                   FastDiv(Wo), FastDiv(Ho));
  else if (k2s2)
    e = launch_pdl(maxpool2x2_fwd_kernel<float>, dim3(grid), dim3(256), 0, st, (const float*)x,
                   (float*)y, idx, planes, H, W, Ho, Wo, FastDiv(Wo), FastDiv(Ho));
  else if (bf16)
    e = launch_pdl(maxpool_fwd_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st,
                   (const __nv_bfloat16*)x, (__nv_bfloat16*)y, idx, planes, H, W, Ho, Wo, g,
                   FastDiv(Wo), FastDiv(Ho));
  else
    e = launch_pdl(maxpool_fwd_kernel<float>, dim3(grid), dim3(256), 0, st, (const float*)x,
                   (float*)y, idx, planes, H, W, Ho, Wo, g, FastDiv(Wo), FastDiv(Ho));
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_maxpool_bwd(const void* dy, bool bf16, const int32_t* idx, void* dx, int planes,
                               int H, int W, int Ho, int Wo, cudaStream_t st) {
  if (planes <= 0 || (int64_t)planes * Ho * Wo >= kMaxFlatIndex) return cudaErrorInvalidValue;
  const int grid = pool_grid((int64_t)planes * Ho * Wo);
  cudaError_t e;
  if (bf16)
    e = launch_pdl(maxpool_bwd_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st,
                   (const __nv_bfloat16*)dy, idx, (__nv_bfloat16*)dx, planes, H * W, Ho * Wo,
                   FastDiv(Ho * Wo));
  else
    e = launch_pdl(maxpool_bwd_kernel<float>, dim3(grid), dim3(256), 0, st, (const float*)dy, idx,
                   (float*)dx, planes, H * W, Ho * Wo, FastDiv(Ho * Wo));
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
