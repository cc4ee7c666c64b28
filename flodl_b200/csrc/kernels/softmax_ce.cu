// Fused softmax cross-entropy (forward loss + gradient in one pass).
//
// Reference: at::cross_entropy_loss with label smoothing and ignore_index
// (flodl-sys/ops_training.cpp:1131-1140, flodl/src/nn/loss.rs). The mean loss
//   L = 1/N * sum_t [ lse_t - (1-eps) z[t,y_t] - eps/V sum_j z[t,j] ]
// and its gradient dz = (softmax(z) - (1-eps) onehot(y) - eps/V) / N are both
// produced here, so backward is a scale (by the upstream scalar) folded into
// the consuming GEMMs. Rows whose target equals ignore_index contribute nothing.
// A target outside [0, V) that is not ignore_index is never used as an index:
// the row is skipped like an ignored one and kErrBadLabel is recorded in the
// error word, which the host reads (the reference's cross-entropy raises).
#include "sm100_ptx.cuh"
#include "kernels.h"

#include <algorithm>

namespace flodl {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_reduce_max(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float r = -INFINITY;
  for (int i = 0; i < kThreads / 32; ++i) r = fmaxf(r, sh[i]);
  return r;
}

__device__ __forceinline__ float block_reduce_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < kThreads / 32; ++i) r += sh[i];
  return r;
}

__device__ __forceinline__ bool target_in_range(int64_t y, int V) { return y >= 0 && y < V; }

// 1 / (number of rows whose target is in [0, V)). One block; every thread
// issues its loads kCountUnroll at a time so the whole target vector is in
// flight at once instead of one dependent load per iteration.
constexpr int kCountThreads = 1024;
constexpr int kCountUnroll = 8;
__global__ void __launch_bounds__(kCountThreads) ce_count_kernel(
    const int64_t* __restrict__ targets, int T, int V, int64_t ignore, float* inv_count,
    float* loss_zero, uint32_t* err) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sh[32];
  float c = 0.f;
  bool bad = false;
  for (int base = threadIdx.x; base < T; base += kCountThreads * kCountUnroll) {
    int64_t y[kCountUnroll];
#pragma unroll
    for (int u = 0; u < kCountUnroll; ++u) {
      const int i = base + u * kCountThreads;
      y[u] = i < T ? __ldg(targets + i) : ignore;
    }
#pragma unroll
    for (int u = 0; u < kCountUnroll; ++u) {
      if (y[u] == ignore) continue;
      if (target_in_range(y[u], V)) c += 1.f;
      else bad = true;
    }
  }
  if (bad) report_error(err, kErrBadLabel);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < kCountThreads / 32; ++i) tot += sh[i];
    *inv_count = tot > 0.f ? 1.f / tot : 0.f;
    if (loss_zero) *loss_zero = 0.f;
  }
}

// Warp per row for vocabularies up to 32 x 8 x NC columns (NC 16-byte chunks
// of 8 bf16 per lane held in registers): one read of the row, shuffle
// reductions, no block barriers. Rows, pitches and V are multiples of 8.
template <int NC>
__global__ void __launch_bounds__(256) softmax_ce_warp_kernel(CeArgs a) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp_g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int n_warps = (gridDim.x * blockDim.x) >> 5;
  const float inv_n = *a.inv_count;
  const float eps = a.smoothing;
  const float off = eps / a.V;
  const int ldd = a.ld_d > 0 ? a.ld_d : a.V;
  float loss_acc = 0.f;
  for (int t = warp_g; t < a.T; t += n_warps) {
    const __nv_bfloat16* z = a.logits + (size_t)t * a.ld;
    const int64_t y = __ldg(a.targets + t);
    const bool valid = (y != a.ignore_index) && target_in_range(y, a.V);
    float v[NC][8];
    float mx = -INFINITY, sz = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < a.V) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(z + col));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16x2(ws[k]);
          v[c][2 * k] = f.x;
          v[c][2 * k + 1] = f.y;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          mx = fmaxf(mx, v[c][k]);
          sz += v[c][k];
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[c][k] = -INFINITY;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      sz += __shfl_xor_sync(0xffffffffu, sz, o);
    }
    float se = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        v[c][k] = __expf(v[c][k] - mx);  // exp(-inf) = 0 past V
        se += v[c][k];
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
    const float inv_se = 1.f / se;
    if (valid && lane == 0) {
      const float zt = __bfloat162float(z[y]);
      loss_acc += (mx + __logf(se) - (1.f - eps) * zt - off * sz) * inv_n;
    }
    if (a.dlogits) {
      __nv_bfloat16* dz = a.dlogits + (size_t)t * ldd;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < a.V) {
          float g[8];
#pragma unroll
          for (int k = 0; k < 8; ++k)
            g[k] = valid ? (v[c][k] * inv_se - off - (col + k == y ? (1.f - eps) : 0.f)) * inv_n
                         : 0.f;
          uint4 w;
          w.x = pack_bf16x2(g[0], g[1]);
          w.y = pack_bf16x2(g[2], g[3]);
          w.z = pack_bf16x2(g[4], g[5]);
          w.w = pack_bf16x2(g[6], g[7]);
          *reinterpret_cast<uint4*>(dz + col) = w;
        }
      }
    }
  }
  // one atomic per block: same-address atomics serialise in L2, one per warp
  // cost more than the whole row pass
  __shared__ float warp_loss[8];
  if (lane == 0) warp_loss[threadIdx.x >> 5] = loss_acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += warp_loss[w];
    if (tot != 0.f) atomicAdd(a.loss, tot);
  }
}

__global__ void __launch_bounds__(kThreads) softmax_ce_kernel(CeArgs a) {
  __shared__ float sh[32];
  const float inv_n = *a.inv_count;
  float loss_acc = 0.f;
  for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
    const __nv_bfloat16* z = a.logits + (size_t)t * a.ld;
    const int64_t y = a.targets[t];
    // out-of-range targets were reported by the count kernel; skip the row
    const bool valid = (y != a.ignore_index) && target_in_range(y, a.V);
    // pass 1: max and sum of logits
    float mx = -INFINITY, sz = 0.f;
    for (int j = threadIdx.x; j < a.V; j += kThreads) {
      float v = __bfloat162float(z[j]);
      mx = fmaxf(mx, v);
      sz += v;
    }
    mx = block_reduce_max(mx, sh);
    sz = block_reduce_sum(sz, sh);
    // pass 2: sum of exp
    float se = 0.f;
    for (int j = threadIdx.x; j < a.V; j += kThreads) se += __expf(__bfloat162float(z[j]) - mx);
    se = block_reduce_sum(se, sh);
    const float lse = mx + __logf(se);
    const float inv_se = 1.f / se;
    const float eps = a.smoothing;
    if (valid && threadIdx.x == 0) {
      const float zt = __bfloat162float(z[y]);
      loss_acc += (lse - (1.f - eps) * zt - eps / a.V * sz) * inv_n;
    }
    if (a.dlogits) {
      __nv_bfloat16* dz = a.dlogits + (size_t)t * (a.ld_d > 0 ? a.ld_d : a.V);
      const float off = eps / a.V;
      for (int j = threadIdx.x; j < a.V; j += kThreads) {
        float g = 0.f;
        if (valid) {
          const float p = __expf(__bfloat162float(z[j]) - mx) * inv_se;
          g = (p - off - (j == y ? (1.f - eps) : 0.f)) * inv_n;
        }
        dz[j] = __float2bfloat16_rn(g);
      }
    }
  }
  if (threadIdx.x == 0 && loss_acc != 0.f) atomicAdd(a.loss, loss_acc);
}

}  // namespace

cudaError_t launch_ce_count(const int64_t* targets, int T, int V, int64_t ignore_index,
                            float* inv_count, float* loss_zero, uint32_t* err, cudaStream_t st) {
  cudaError_t le = launch_pdl(ce_count_kernel, dim3(1), dim3(kCountThreads), 0, st, targets, T, V,
                              ignore_index, inv_count, loss_zero,
                              err ? err : default_err_word());
  if (le != cudaSuccess) return le;
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_softmax_ce(const CeArgs& a, cudaStream_t st) {
  if (a.T <= 0 || a.V <= 0) return cudaErrorInvalidValue;
  const int ldd = a.ld_d > 0 ? a.ld_d : a.V;
  const bool aligned = a.V % 8 == 0 && a.ld % 8 == 0 && ldd % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(a.logits) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(a.dlogits) & 15) == 0;
  if (aligned && a.V <= 32 * 8 * 8) {
    // warp per row; 32 warps per SM (a few rows each), 8 warps per block
    const int nc = (a.V + 255) / 256;
    const int64_t warps = std::min<int64_t>(a.T, (int64_t)num_sms() * 32);
    const int grid = (int)((warps * 32 + 255) / 256);
    cudaError_t e = cudaSuccess;
    switch (nc) {
      case 1: e = launch_pdl(softmax_ce_warp_kernel<1>, dim3(grid), dim3(256), 0, st, a); break;
      case 2: e = launch_pdl(softmax_ce_warp_kernel<2>, dim3(grid), dim3(256), 0, st, a); break;
      case 3: case 4:
        e = launch_pdl(softmax_ce_warp_kernel<4>, dim3(grid), dim3(256), 0, st, a);
        break;
      default: e = launch_pdl(softmax_ce_warp_kernel<8>, dim3(grid), dim3(256), 0, st, a); break;
    }
    if (e != cudaSuccess) return e;
    note_launch();
    return cudaGetLastError();
  }
  int grid = a.T < num_sms() * 8 ? a.T : num_sms() * 8;
  softmax_ce_kernel<<<grid, kThreads, 0, st>>>(a);
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
