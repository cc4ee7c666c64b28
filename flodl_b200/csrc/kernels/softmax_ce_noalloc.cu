// Allocation-free C entry point for the fused softmax cross-entropy.
//
// This entry point has no counterpart in the reference (fab2s/floDl); it is an
// addition of this library.
//
// Who it is for: callers that cannot call cudaMalloc (or any allocating
// routine) at the point where they need the loss. Typical cases are code that
// runs while another component owns the device's memory budget and forbids
// new allocations (a fixed-pool serving runtime, an embedded plug-in that may
// only use memory handed to it), and host code inside a context where an
// allocation would synchronise the device or fail (for example while a
// memory pool is being resized elsewhere). The regular entry point
// (`softmax_ce` in the torch bindings) needs a caller-allocated scratch word
// for the 1/count factor; this one keeps its scratch in a fixed device array
// instead, so the caller passes only its inputs and outputs.
//
// Contract:
//  * Scratch: a file-scope device array of kNoAllocMaxRows + 64 floats
//    (about 1 MiB). Every GPU that loads this library holds it until the
//    process exits. Rows beyond kNoAllocMaxRows are rejected with
//    FLODL_NOALLOC_ERR_TOO_MANY_ROWS; nothing is launched in that case.
//  * Set-up: the first call on a device (with that device current) looks up
//    the array's device address with cudaGetSymbolAddress and caches it for
//    that device. Make that first call before any stream capture begins.
//  * Every call on a device shares the same array and leaves the last call's
//    contents in it. All scratch slots a call reads are written earlier in
//    the same call (the count and the bad-row count, then one loss per row,
//    ignored rows as 0), so nothing has to start at zero.
//  * A target outside [0, V) that is not ignore_index is never used as an
//    index: that row is skipped like an ignored one and counted in scratch
//    slot 1, which flodl_softmax_ce_noalloc_bad_rows reads back.
//  * Calls that overlap on the GPU (different streams, or a second call
//    launched before the first finished on another stream) race on the
//    array; serialise them on one stream.
//  * The mean loss is the deterministic sum of per-row losses (no atomics);
//    dlogits (nullable) receives the gradient of the mean loss, as the
//    regular entry point writes it.
//  * No cudaMalloc, cudaFree or other allocating routine is called.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "softmax_ce_noalloc.h"

namespace {

constexpr int kNoAllocMaxRows = 262144;  // rows (tokens) per call
constexpr int kScratchHeader = 64;       // floats: [0] = 1/count, [1] = bad rows (u32 bits)
constexpr int kMaxDevices = 64;
constexpr int kThreads = 256;

static __device__ __align__(256) float g_ce_noalloc_scratch[kScratchHeader + kNoAllocMaxRows];

struct DeviceSetup {
  float* scratch = nullptr;  // device address of g_ce_noalloc_scratch on this device
  int sms = 0;               // multiprocessor count of this device
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mu;

__device__ __forceinline__ bool target_in_range(int64_t y, int V) { return y >= 0 && y < V; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < (int)(blockDim.x / 32); ++i) r += sh[i];
  return r;
}
__device__ float block_max(float v, float* sh) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = -INFINITY;
  for (int i = 0; i < (int)(blockDim.x / 32); ++i) r = fmaxf(r, sh[i]);
  return r;
}

// scratch[0] = 1 / number of rows whose target is in [0, V);
// scratch[1] = number of rows whose target is out of range and not ignore_index
__global__ void noalloc_count_kernel(const int64_t* __restrict__ targets, int T, int V,
                                     int64_t ignore, float* scratch) {
  __shared__ float sh[32];
  float c = 0.f, bad = 0.f;
  for (int i = threadIdx.x; i < T; i += blockDim.x) {
    const int64_t y = targets[i];
    if (y == ignore) continue;
    if (target_in_range(y, V)) c += 1.f;
    else bad += 1.f;
  }
  const float tot = block_sum(c, sh);
  const float nbad = block_sum(bad, sh);
  if (threadIdx.x == 0) {
    scratch[0] = tot > 0.f ? 1.f / tot : 0.f;
    reinterpret_cast<uint32_t*>(scratch)[1] = (uint32_t)nbad;
  }
}

// scratch[kScratchHeader + t] = loss of row t / count (0 for ignored rows)
__global__ void __launch_bounds__(kThreads)
    noalloc_rows_kernel(const __nv_bfloat16* __restrict__ logits, int ld,
                        const int64_t* __restrict__ targets, int T, int V, int64_t ignore,
                        float smoothing, float* scratch, __nv_bfloat16* __restrict__ dlogits) {
  __shared__ float sh[32];
  const float inv_n = scratch[0];
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    const __nv_bfloat16* z = logits + (size_t)t * ld;
    const int64_t y = targets[t];
    const bool valid = (y != ignore) && target_in_range(y, V);  // z[y] is read only when valid
    float mx = -INFINITY, sz = 0.f;
    for (int j = threadIdx.x; j < V; j += kThreads) {
      const float v = __bfloat162float(z[j]);
      mx = fmaxf(mx, v);
      sz += v;
    }
    mx = block_max(mx, sh);
    sz = block_sum(sz, sh);
    float se = 0.f;
    for (int j = threadIdx.x; j < V; j += kThreads) se += __expf(__bfloat162float(z[j]) - mx);
    se = block_sum(se, sh);
    const float lse = mx + __logf(se);
    if (threadIdx.x == 0) {
      float l = 0.f;
      if (valid) {
        const float zt = __bfloat162float(z[y]);
        l = (lse - (1.f - smoothing) * zt - smoothing / V * sz) * inv_n;
      }
      scratch[kScratchHeader + t] = l;
    }
    if (dlogits) {
      __nv_bfloat16* dz = dlogits + (size_t)t * V;
      const float inv_se = 1.f / se;
      const float off = smoothing / V;
      for (int j = threadIdx.x; j < V; j += kThreads) {
        float g = 0.f;
        if (valid) {
          const float p = __expf(__bfloat162float(z[j]) - mx) * inv_se;
          g = (p - off - (j == y ? (1.f - smoothing) : 0.f)) * inv_n;
        }
        dz[j] = __float2bfloat16_rn(g);
      }
    }
  }
}

// *loss_out = sum of the per-row losses (fixed order within a single block)
__global__ void noalloc_reduce_kernel(const float* __restrict__ scratch, int T, float* loss_out) {
  __shared__ float sh[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < T; i += blockDim.x) s += scratch[kScratchHeader + i];
  const float tot = block_sum(s, sh);
  if (threadIdx.x == 0) *loss_out = tot;
}

// Looks up (once per device, with that device current) the device address of
// the scratch array and the device's multiprocessor count.
cudaError_t setup_for_current_device(DeviceSetup* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  DeviceSetup& s = g_setup[dev];
  if (s.scratch == nullptr) {
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    if (sms <= 0) return cudaErrorInvalidDevice;
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ce_noalloc_scratch);
    if (e != cudaSuccess) return e;
    s.sms = sms;
    s.scratch = static_cast<float*>(p);
  }
  *out = s;
  return cudaSuccess;
}

}  // namespace

// Arguments and return codes: softmax_ce_noalloc.h. Returns 0 on success,
// FLODL_NOALLOC_ERR_TOO_MANY_ROWS when T exceeds the fixed scratch capacity
// (262144 rows), FLODL_NOALLOC_ERR_BAD_ARGS for invalid sizes or null
// pointers, or a positive cudaError_t value.
extern "C" __attribute__((visibility("default"))) int flodl_softmax_ce_noalloc(
    const void* logits, int ld, const int64_t* targets, int T, int V, int64_t ignore_index,
    float smoothing, float* loss_out, void* dlogits, cudaStream_t stream) {
  if (T <= 0 || V <= 0 || ld < V || !logits || !targets || !loss_out)
    return FLODL_NOALLOC_ERR_BAD_ARGS;
  if (T > kNoAllocMaxRows) return FLODL_NOALLOC_ERR_TOO_MANY_ROWS;
  DeviceSetup dev;
  cudaError_t e = setup_for_current_device(&dev);
  if (e != cudaSuccess) return (int)e;
  float* scratch = dev.scratch;
  noalloc_count_kernel<<<1, kThreads, 0, stream>>>(targets, T, V, ignore_index, scratch);
  const int grid = T < dev.sms * 8 ? T : dev.sms * 8;
  noalloc_rows_kernel<<<grid, kThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(logits), ld, targets, T, V, ignore_index, smoothing,
      scratch, static_cast<__nv_bfloat16*>(dlogits));
  noalloc_reduce_kernel<<<1, 1024, 0, stream>>>(scratch, T, loss_out);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

// Capacity of the fixed scratch array, in rows.
extern "C" __attribute__((visibility("default"))) int flodl_softmax_ce_noalloc_max_rows(void) {
  return kNoAllocMaxRows;
}

// Bad-row count of the last call on the current device (scratch slot 1).
extern "C" __attribute__((visibility("default"))) int flodl_softmax_ce_noalloc_bad_rows(
    cudaStream_t stream, int* out) {
  if (!out) return FLODL_NOALLOC_ERR_BAD_ARGS;
  DeviceSetup dev;
  cudaError_t e = setup_for_current_device(&dev);
  if (e != cudaSuccess) return (int)e;
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return (int)e;
  uint32_t v = 0;
  e = cudaMemcpy(&v, reinterpret_cast<const uint32_t*>(dev.scratch) + 1, sizeof(v),
                 cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return (int)e;
  *out = (int)v;
  return 0;
}
