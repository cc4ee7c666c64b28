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

__global__ void ce_count_kernel(const int64_t* __restrict__ targets, int T, int V, int64_t ignore,
                                float* inv_count, float* loss_zero, uint32_t* err) {
  __shared__ float sh[32];
  float c = 0.f;
  bool bad = false;
  for (int i = threadIdx.x; i < T; i += blockDim.x) {
    const int64_t y = targets[i];
    if (y == ignore) continue;
    if (target_in_range(y, V)) c += 1.f;
    else bad = true;
  }
  if (bad) report_error(err, kErrBadLabel);
  float tot = block_reduce_sum(c, sh);
  if (threadIdx.x == 0) {
    *inv_count = tot > 0.f ? 1.f / tot : 0.f;
    if (loss_zero) *loss_zero = 0.f;
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
  ce_count_kernel<<<1, kThreads, 0, st>>>(targets, T, V, ignore_index, inv_count, loss_zero,
                                          err ? err : default_err_word());
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_softmax_ce(const CeArgs& a, cudaStream_t st) {
  if (a.T <= 0 || a.V <= 0) return cudaErrorInvalidValue;
  int grid = a.T < num_sms() * 8 ? a.T : num_sms() * 8;
  softmax_ce_kernel<<<grid, kThreads, 0, st>>>(a);
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
