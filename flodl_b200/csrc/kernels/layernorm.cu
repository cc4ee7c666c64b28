// Fused LayerNorm forward/backward for sm_100a (memory-bound, one warp per row).
//
// Forward (reference: at::native_layer_norm, flodl-sys/ops_tensor.cpp:580-600):
//   y = (x - mean) * rstd * gamma + beta,  rstd = 1/sqrt(var + eps)
//   x is the f32 (or bf16) residual stream; y is written in bf16 so it feeds the
//   tcgen05 GEMM directly (or in f32), mean/rstd are kept for backward.
//
// Backward, fused in one pass over the rows:
//   dx    = rstd * (g - mean(g) - xhat * mean(g * xhat)),  g = dy * gamma
//   dx   += dres                         (gradient arriving on the skip path)
//   dgamma += sum_rows dy * xhat,  dbeta += sum_rows dy     (f32, atomics per block)
//   colsum += sum_rows dx                (bias gradient of the Linear whose output
//                                         was added into this residual stream)
//   dx is written in f32 (the residual chain) and/or bf16 (the GEMM operand).
#include "sm100_ptx.cuh"
#include "kernels.h"

#include <algorithm>
#include <atomic>
#include <mutex>
#include <set>
#include <utility>

namespace flodl {

namespace {

template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&v)[4]) {
  float4 f = *reinterpret_cast<const float4*>(p);
  v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

__device__ __forceinline__ void store4_bf16(__nv_bfloat16* p, const float (&v)[4]) {
  uint2 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ void store4_f32(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kWarps = 8;

// cp.async staging for the backward pass: each lane copies its own column
// chunks of the next row into its warp's shared-memory slot and later reads
// back only what it copied itself, so no warp barrier is needed - only the
// per-thread cp.async group wait.
__device__ __forceinline__ void cp_async_8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
template <typename T>
__device__ __forceinline__ void cp_async_4elems(void* dst, const T* src);
template <>
__device__ __forceinline__ void cp_async_4elems<float>(void* dst, const float* src) {
  cp_async_16(dst, src);
}
template <>
__device__ __forceinline__ void cp_async_4elems<__nv_bfloat16>(void* dst, const __nv_bfloat16* src) {
  cp_async_8(dst, src);
}
template <typename T>
__device__ __forceinline__ void lds4(const uint8_t* p, float (&v)[4]);
template <>
__device__ __forceinline__ void lds4<float>(const uint8_t* p, float (&v)[4]) {
  const float4 f = *reinterpret_cast<const float4*>(p);
  v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
}
template <>
__device__ __forceinline__ void lds4<__nv_bfloat16>(const uint8_t* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
// Rows up to kStagedMaxNV * 128 columns take the staged path; one slot holds
// x, dy and the skip-path gradient of one row for one warp.
constexpr int kStagedMaxNV = 4;
template <typename TIn, int NV>
struct LnBwdSlot {
  static constexpr int kX = 4 * (int)sizeof(TIn);  // bytes per lane chunk
  static constexpr int kXOff = 0;
  static constexpr int kDyOff = NV * 32 * kX;
  static constexpr int kROff = kDyOff + NV * 32 * 8;
  static constexpr int kBytes = kROff + NV * 32 * 16;
  static constexpr int kBlockBytes = NV <= kStagedMaxNV ? kWarps * 2 * kBytes : 0;
};

// NV = number of 128-element column groups (C <= NV*128); lane owns columns
// lane*4 + 128*j .. +3 for j < NV.
template <typename TIn, int NV>
__global__ void __launch_bounds__(kWarps * 32, NV <= 4 ? 4 : 1) ln_fwd_kernel(
    const TIn* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    __nv_bfloat16* __restrict__ y_bf16, float* __restrict__ y_f32, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int rows, int C, float eps) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp_global = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * kWarps;
  // gamma/beta are read per row through the read-only cache (L1-resident):
  // holding them in registers cost a quarter of the resident warps.
  for (int r = warp_global; r < rows; r += nwarps) {
    const TIn* xr = x + (size_t)r * C;
    float v[NV][4];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = lane * 4 + 128 * j;
      if (c < C) {
        load4<TIn>(xr + c, v[j]);
      } else {
        v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.f;
      }
      s += v[j][0] + v[j][1] + v[j][2] + v[j][3];
    }
    const float mean = warp_sum(s) / C;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = lane * 4 + 128 * j;
      if (c < C) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float d = v[j][e] - mean;
          ss += d * d;
        }
      }
    }
    const float rstd = rsqrtf(warp_sum(ss) / C + eps);
    if (lane == 0) {
      if (mean_out) mean_out[r] = mean;
      if (rstd_out) rstd_out[r] = rstd;
    }
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = lane * 4 + 128 * j;
      if (c < C) {
        const float4 g4 = gamma ? __ldg(reinterpret_cast<const float4*>(gamma + c))
                                : make_float4(1.f, 1.f, 1.f, 1.f);
        const float4 b4 = beta ? __ldg(reinterpret_cast<const float4*>(beta + c))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = (v[j][e] - mean) * rstd * gv[e] + bv[e];
        if (y_bf16) store4_bf16(y_bf16 + (size_t)r * C + c, o);
        if (y_f32) store4_f32(y_f32 + (size_t)r * C + c, o);
      }
    }
  }
}

template <typename TIn, int NV>
__global__ void __launch_bounds__(kWarps * 32, 2) ln_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const TIn* __restrict__ x,
    const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
    const float* __restrict__ gamma, const float* __restrict__ dres, float* __restrict__ dx_f32,
    __nv_bfloat16* __restrict__ dx_bf16, float* __restrict__ dgamma, float* __restrict__ dbeta,
    float* __restrict__ colsum, int rows, int C, float* __restrict__ partials, int pre_add) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int warp_global = blockIdx.x * kWarps + wib;
  const int nwarps = gridDim.x * kWarps;
  float acc_dg[NV][4], acc_db[NV][4], acc_cs[NV][4];
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc_dg[j][e] = acc_db[j][e] = acc_cs[j][e] = 0.f;
  using Slot = LnBwdSlot<TIn, NV>;
  constexpr bool kStaged = NV <= kStagedMaxNV;
  extern __shared__ __align__(16) uint8_t ln_stage[];
  uint8_t* wslots = ln_stage + (size_t)wib * 2 * Slot::kBytes;
  // the next row of this warp goes into the other slot while this one is used
  auto stage_row = [&](int r, int slot) {
    uint8_t* b = wslots + slot * Slot::kBytes;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = lane * 4 + 128 * j;
      const int k = j * 32 + lane;
      if (c < C) {
        cp_async_4elems<TIn>(b + Slot::kXOff + k * Slot::kX, x + (size_t)r * C + c);
        cp_async_8(b + Slot::kDyOff + k * 8, dy + (size_t)r * C + c);
        if (dres) cp_async_16(b + Slot::kROff + k * 16, dres + (size_t)r * C + c);
      }
    }
    cp_async_commit();  // every lane commits, copies or not: group counts stay uniform
  };
  int slot = 0;
  if (kStaged && warp_global < rows) stage_row(warp_global, 0);
  for (int r = warp_global; r < rows; r += nwarps, slot ^= 1) {
    float xh[NV][4], dyv[NV][4], rv[NV][4];
    if constexpr (kStaged) {
      if (r + nwarps < rows) {
        stage_row(r + nwarps, slot ^ 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      const uint8_t* b = wslots + slot * Slot::kBytes;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = lane * 4 + 128 * j;
        const int k = j * 32 + lane;
        if (c < C) {
          lds4<TIn>(b + Slot::kXOff + k * Slot::kX, xh[j]);
          lds4<__nv_bfloat16>(b + Slot::kDyOff + k * 8, dyv[j]);
          if (dres) lds4<float>(b + Slot::kROff + k * 16, rv[j]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) xh[j][e] = dyv[j][e] = 0.f;
        }
      }
    } else {
      // issue every load of the row up front (x, dy, skip-path gradient)
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = lane * 4 + 128 * j;
        if (c < C) {
          load4<TIn>(x + (size_t)r * C + c, xh[j]);
          load4<__nv_bfloat16>(dy + (size_t)r * C + c, dyv[j]);
          if (dres) load4<float>(dres + (size_t)r * C + c, rv[j]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) xh[j][e] = dyv[j][e] = 0.f;
        }
      }
    }
    if (pre_add && dres) {
      // post-LN blocks: the LayerNorm's output gradient is dy + dres
#pragma unroll
      for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) dyv[j][e] += rv[j][e];
    }
    const float mean = mean_in[r];
    const float rstd = rstd_in[r];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = lane * 4 + 128 * j;
      if (c < C) {
        const float4 g4 = gamma ? __ldg(reinterpret_cast<const float4*>(gamma + c))
                                : make_float4(1.f, 1.f, 1.f, 1.f);
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xh[j][e] = (xh[j][e] - mean) * rstd;
          const float gg = dyv[j][e] * gv[e];
          s1 += gg;
          s2 += gg * xh[j][e];
          acc_dg[j][e] += dyv[j][e] * xh[j][e];
          acc_db[j][e] += dyv[j][e];
          dyv[j][e] = gg;  // keep dy * gamma
        }
      }
    }
    const float m1 = warp_sum(s1) / C;
    const float m2 = warp_sum(s2) / C;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = lane * 4 + 128 * j;
      if (c < C) {
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o[e] = rstd * (dyv[j][e] - m1 - xh[j][e] * m2);
          if (dres && !pre_add) o[e] += rv[j][e];
          acc_cs[j][e] += o[e];
        }
        if (dx_f32) store4_f32(dx_f32 + (size_t)r * C + c, o);
        if (dx_bf16) store4_bf16(dx_bf16 + (size_t)r * C + c, o);
      }
    }
  }
  // Block reduction of the per-column partials. With `partials`, each block
  // writes its three C-wide partial rows there (slot k of block b at
  // partials[(k * gridDim.x + b) * C]) for a deterministic second pass;
  // otherwise one atomic per column.
  __shared__ float red[kWarps][128];
  auto flush = [&](float (&acc)[NV][4], float* out, int k) {
    if (!out) return;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) red[wib][lane * 4 + e] = acc[j][e];
      __syncthreads();
      if (threadIdx.x < 128) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[w][threadIdx.x];
        const int c = threadIdx.x + 128 * j;
        if (c < C) {
          if (partials)
            partials[((size_t)k * gridDim.x + blockIdx.x) * C + c] = s;
          else
            atomicAdd(out + c, s);
        }
      }
      __syncthreads();
    }
  };
  flush(acc_dg, dgamma, 0);
  flush(acc_db, dbeta, 1);
  flush(acc_cs, colsum, 2);
}

// Second pass of the two-stage column reductions: out[c] += sum_b partials[b][c]
// for up to three (partials, out) pairs laid out as [k][nblocks][C]. Block =
// 32 columns x 8 partial lanes; each thread keeps four independent sums.
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ partials,
                                                              int nblocks, int C, float* out0,
                                                              float* out1, float* out2,
                                                              const float* __restrict__ scale) {
  const int c = blockIdx.x * 32 + threadIdx.x;
  const int k = blockIdx.y;
  float* out = k == 0 ? out0 : (k == 1 ? out1 : out2);
  if (out == nullptr) return;  // uniform across the block
  const float* p = partials + (size_t)k * nblocks * C;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (c < C) {
    int b = threadIdx.y;
    for (; b + 24 < nblocks; b += 32) {
      s0 += p[(size_t)b * C + c];
      s1 += p[(size_t)(b + 8) * C + c];
      s2 += p[(size_t)(b + 16) * C + c];
      s3 += p[(size_t)(b + 24) * C + c];
    }
    for (; b < nblocks; b += 8) s0 += p[(size_t)b * C + c];
  }
  __shared__ float red[8][33];
  red[threadIdx.y][threadIdx.x] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (threadIdx.y == 0 && c < C) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x];
    if (scale) t *= *scale;
    out[c] += t;
  }
}

// Column sums, first pass: block b sums rows [b*R, (b+1)*R) of a [rows, C]
// matrix; thread owns 8 consecutive columns (16-byte loads), several row
// lanes per block when C is narrow. Writes partials[b][c].
template <typename T, int NT>
__global__ void __launch_bounds__(NT) colsum_partial_kernel(const T* __restrict__ m,
                                                             float* __restrict__ partials,
                                                             int rows, int C, int rows_per_block,
                                                             float* __restrict__ out,
                                                             const float* __restrict__ scale) {
  const int groups = C / 8;                       // 8-column groups per row
  const int tpr = groups < 256 ? groups : 256;    // threads per row slice
  const int lanes = NT / tpr;                     // row slices per block
  const int g0 = blockIdx.y * 256;                // column-group offset of this block
  const int tid = threadIdx.x;
  const int gi = g0 + (tid % tpr);
  const int slice = tid / tpr;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  if (slice < lanes && gi < groups) {
#pragma unroll 8
    for (int r = r0 + slice; r < r1; r += lanes) {
      const T* src = m + (size_t)r * C + gi * 8;
      float v[8];
      if constexpr (sizeof(T) == 2) {
        uint4 u = *reinterpret_cast<const uint4*>(src);
        float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c2 = unpack_bf16x2(u.z),
               d = unpack_bf16x2(u.w);
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c2.x; v[5] = c2.y; v[6] = d.x; v[7] = d.y;
      } else {
        float4 a = *reinterpret_cast<const float4*>(src);
        float4 b = *reinterpret_cast<const float4*>(src + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += v[e];
    }
  }
  __shared__ float red[NT][9];
#pragma unroll
  for (int e = 0; e < 8; ++e) red[tid][e] = acc[e];
  __syncthreads();
  if (slice == 0 && gi < groups) {
    for (int l = 1; l < lanes; ++l)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += red[tid + l * tpr][e];
    if (partials) {
#pragma unroll
      for (int e = 0; e < 8; ++e) partials[(size_t)blockIdx.x * C + gi * 8 + e] = acc[e];
    } else {
      // single pass: one atomic per column and block
      const float sc = scale ? __ldg(scale) : 1.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) atomicAdd(out + gi * 8 + e, acc[e] * sc);
    }
  }
}

// Column sums of a [rows, C] matrix into f32 out[C] (accumulating).
template <typename T>
__global__ void colsum_kernel(const T* __restrict__ m, float* __restrict__ out, int rows, int C,
                              int rows_per_block, const float* __restrict__ scale, int ld) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  float s = 0.f;
  for (int r = r0; r < r1; ++r) s += to_f32(m[(size_t)r * ld + c]);
  if (scale) s *= *scale;
  atomicAdd(out + c, s);
}

int grid_for_rows(int rows) {
  int blocks = (rows + kWarps - 1) / kWarps;
  int cap = num_sms() * 8;
  return blocks < cap ? blocks : cap;
}

}  // namespace

// Dynamic shared memory above the 48 KB default needs a per-device,
// per-function opt-in; done once per (function, device).
static cudaError_t opt_in_smem(const void* fn, int bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({fn, dev})) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert({fn, dev});
  return e;
}

#define FL_LN_DISPATCH_NV(C, ...) \
  do {                                   \
    int nv_ = ((C) + 127) / 128;         \
    if (nv_ <= 1) { constexpr int NV = 1; __VA_ARGS__; } \
    else if (nv_ <= 2) { constexpr int NV = 2; __VA_ARGS__; } \
    else if (nv_ <= 4) { constexpr int NV = 4; __VA_ARGS__; } \
    else if (nv_ <= 6) { constexpr int NV = 6; __VA_ARGS__; } \
    else if (nv_ <= 8) { constexpr int NV = 8; __VA_ARGS__; } \
    else if (nv_ <= 16) { constexpr int NV = 16; __VA_ARGS__; } \
    else return cudaErrorInvalidValue;   \
  } while (0)

// One wave of resident blocks: the grid is capped at what the SMs hold at
// once (occupancy of this kernel instance, cached per device), and each warp
// strides over its rows. A grid of 1.6 waves left the second wave's SMs
// partly idle.
template <typename Kern>
static int resident_grid(Kern kern, int rows, std::atomic<int>& cache) {
  int per_sm = cache.load(std::memory_order_relaxed);
  if (per_sm <= 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarps * 32, 0) !=
            cudaSuccess ||
        per_sm <= 0)
      per_sm = 2;
    cache.store(per_sm, std::memory_order_relaxed);
  }
  const int blocks = (rows + kWarps - 1) / kWarps;
  const int cap = num_sms() * per_sm;
  return blocks < cap ? blocks : cap;
}

cudaError_t launch_ln_fwd(const LnFwdArgs& a, cudaStream_t st) {
  if (a.C % 4 != 0) return cudaErrorInvalidValue;
  if (a.x_bf16) {
    FL_LN_DISPATCH_NV(a.C, {
      auto k = ln_fwd_kernel<__nv_bfloat16, NV>;
      static std::atomic<int> occ{0};
      cudaError_t le = launch_pdl(k, dim3(resident_grid(k, a.rows, occ)), dim3(kWarps * 32), 0, st,
                                  (const __nv_bfloat16*)a.x, a.gamma, a.beta, a.y_bf16, a.y_f32,
                                  a.mean, a.rstd, a.rows, a.C, a.eps);
      if (le != cudaSuccess) return le;
    });
  } else {
    FL_LN_DISPATCH_NV(a.C, {
      auto k = ln_fwd_kernel<float, NV>;
      static std::atomic<int> occ{0};
      cudaError_t le = launch_pdl(k, dim3(resident_grid(k, a.rows, occ)), dim3(kWarps * 32), 0, st,
                                  (const float*)a.x, a.gamma, a.beta, a.y_bf16, a.y_f32, a.mean,
                                  a.rstd, a.rows, a.C, a.eps);
      if (le != cudaSuccess) return le;
    });
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_ln_bwd(const LnBwdArgs& a, cudaStream_t st) {
  if (a.C % 4 != 0) return cudaErrorInvalidValue;
  // with partials: two deterministic passes; without: one pass, one atomic
  // per column and block (grid capped at two blocks per SM)
  const int grid = a.partials ? a.partial_blocks : std::min(grid_for_rows(a.rows), num_sms() * 2);
  if (a.x_bf16) {
    FL_LN_DISPATCH_NV(a.C, {
      auto k = ln_bwd_kernel<__nv_bfloat16, NV>;
      constexpr int smem = LnBwdSlot<__nv_bfloat16, NV>::kBlockBytes;
      cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(k), smem);
      if (e != cudaSuccess) return e;
      e = launch_pdl(k, dim3(grid), dim3(kWarps * 32), smem, st, a.dy, (const __nv_bfloat16*)a.x,
                     (const float*)a.mean, (const float*)a.rstd, a.gamma, a.dres, a.dx_f32,
                     a.dx_bf16, a.dgamma, a.dbeta, a.colsum, a.rows, a.C, a.partials,
                     a.pre_add ? 1 : 0);
      if (e != cudaSuccess) return e;
    });
  } else {
    FL_LN_DISPATCH_NV(a.C, {
      auto k = ln_bwd_kernel<float, NV>;
      constexpr int smem = LnBwdSlot<float, NV>::kBlockBytes;
      cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(k), smem);
      if (e != cudaSuccess) return e;
      e = launch_pdl(k, dim3(grid), dim3(kWarps * 32), smem, st, a.dy, (const float*)a.x,
                     (const float*)a.mean, (const float*)a.rstd, a.gamma, a.dres, a.dx_f32,
                     a.dx_bf16, a.dgamma, a.dbeta, a.colsum, a.rows, a.C, a.partials,
                     a.pre_add ? 1 : 0);
      if (e != cudaSuccess) return e;
    });
  }
  note_launch();
  if (a.partials) {
    dim3 rg((a.C + 31) / 32, 3);
    reduce_partials_kernel<<<rg, dim3(32, 8), 0, st>>>(a.partials, grid, a.C, a.dgamma, a.dbeta,
                                                       a.colsum, nullptr);
    note_launch();
  }
  return cudaGetLastError();
}

int ln_bwd_partial_blocks(int rows) { return grid_for_rows(rows) < num_sms() * 4 ? grid_for_rows(rows) : num_sms() * 4; }

int colsum_partial_blocks(int rows) {
  // one row slice per SM: enough loads in flight (8-deep unrolled) to stream
  // at HBM speed, and only num_sms atomics per column in the single-pass mode
  int b = num_sms();
  return rows < b ? (rows > 0 ? rows : 1) : b;
}

cudaError_t launch_colsum2(const void* m, bool bf16, float* out, int rows, int C, float* partials,
                           int nblocks, cudaStream_t st, const float* scale) {
  if (C % 8 != 0) return launch_colsum(m, bf16, out, rows, C, st, scale);
  const int rpb = (rows + nblocks - 1) / nblocks;
  dim3 g1(nblocks, (C / 8 + 255) / 256);
  if (bf16)
    colsum_partial_kernel<__nv_bfloat16, 256><<<g1, 256, 0, st>>>(
        (const __nv_bfloat16*)m, partials, rows, C, rpb, nullptr, nullptr);
  else
    colsum_partial_kernel<float, 256><<<g1, 256, 0, st>>>((const float*)m, partials, rows, C, rpb,
                                                          nullptr, nullptr);
  dim3 g2((C + 31) / 32, 1);
  reduce_partials_kernel<<<g2, dim3(32, 8), 0, st>>>(partials, nblocks, C, out, nullptr, nullptr,
                                                     scale);
  note_launch(2);
  return cudaGetLastError();
}

cudaError_t launch_colsum_atomic(const void* m, bool bf16, float* out, int rows, int C,
                                 int nblocks, cudaStream_t st, const float* scale) {
  if (C % 8 != 0) return launch_colsum(m, bf16, out, rows, C, st, scale);
  const int rpb = (rows + nblocks - 1) / nblocks;
  dim3 g1(nblocks, (C / 8 + 255) / 256);
  if (bf16)
    colsum_partial_kernel<__nv_bfloat16, 1024><<<g1, 1024, 0, st>>>(
        (const __nv_bfloat16*)m, nullptr, rows, C, rpb, out, scale);
  else
    colsum_partial_kernel<float, 1024><<<g1, 1024, 0, st>>>((const float*)m, nullptr, rows, C, rpb,
                                                            out, scale);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_colsum(const void* m, bool bf16, float* out, int rows, int C, cudaStream_t st,
                          const float* scale, int ld) {
  if (ld <= 0) ld = C;
  const int threads = 128;
  const int rows_per_block = 256;
  dim3 grid((C + threads - 1) / threads, (rows + rows_per_block - 1) / rows_per_block);
  if (bf16)
    colsum_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>((const __nv_bfloat16*)m, out, rows, C,
                                                           rows_per_block, scale, ld);
  else
    colsum_kernel<float><<<grid, threads, 0, st>>>((const float*)m, out, rows, C, rows_per_block,
                                                   scale, ld);
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
