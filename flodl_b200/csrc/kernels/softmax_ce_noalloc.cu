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
//    the same call (the count, then one loss per row, ignored rows as 0), so
//    nothing has to start at zero. Calls that overlap on the GPU (different
//    streams, or a second call launched before the first finished on another
//    stream) race on the array; serialise them on one stream.
//  * The mean loss is the deterministic sum of per-row losses (no atomics);
//    dlogits (nullable) receives the gradient of the mean loss, as the
//    regular entry point writes it.
//  * No cudaMalloc, cudaFree or other allocating routine is called.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace {

constexpr int kNoAllocMaxRows = 262144;  // rows (tokens) per call
constexpr int kScratchHeader = 64;       // floats: [0] = 1/count, rest reserved
constexpr int kMaxDevices = 64;
constexpr int kThreads = 256;

static __device__ __align__(256) float g_ce_noalloc_scratch[kScratchHeader + kNoAllocMaxRows];

float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_setup_mu;

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

// scratch[0] = 1 / number of rows whose target is not ignore_index
__global__ void noalloc_count_kernel(const int64_t* __restrict__ targets, int T, int64_t ignore,
                                     float* scratch) {
  __shared__ float sh[32];
  float c = 0.f;
  for (int i = threadIdx.x; i < T; i += blockDim.x) c += (targets[i] != ignore) ? 1.f : 0.f;
  const float tot = block_sum(c, sh);
  if (threadIdx.x == 0) scratch[0] = tot > 0.f ? 1.f / tot : 0.f;
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
    const bool valid = (y != ignore);
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

// Looks up (once per device) the device address of the scratch array.
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ce_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

#define FLODL_NOALLOC_ERR_TOO_MANY_ROWS (-1)
#define FLODL_NOALLOC_ERR_BAD_ARGS (-2)

// Fused softmax cross-entropy that allocates nothing.
//   logits   : bf16 [T, V], row pitch `ld` elements (device)
//   targets  : int64 [T] (device); rows equal to ignore_index are skipped
//   loss_out : f32 scalar (device), receives the mean loss
//   dlogits  : bf16 [T, V] contiguous (device) or NULL, receives d(mean loss)/dlogits
//   stream   : CUDA stream to launch on (0 = legacy default stream)
// Returns 0 on success, FLODL_NOALLOC_ERR_TOO_MANY_ROWS when T exceeds the
// fixed scratch capacity (262144 rows), FLODL_NOALLOC_ERR_BAD_ARGS for invalid
// sizes or null pointers, or a positive cudaError_t value.
extern "C" __attribute__((visibility("default"))) int flodl_softmax_ce_noalloc(
    const void* logits, int ld, const int64_t* targets, int T, int V, int64_t ignore_index,
    float smoothing, float* loss_out, void* dlogits, cudaStream_t stream) {
  if (T <= 0 || V <= 0 || ld < V || !logits || !targets || !loss_out)
    return FLODL_NOALLOC_ERR_BAD_ARGS;
  if (T > kNoAllocMaxRows) return FLODL_NOALLOC_ERR_TOO_MANY_ROWS;
  float* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return (int)e;
  noalloc_count_kernel<<<1, kThreads, 0, stream>>>(targets, T, ignore_index, scratch);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = T < sms * 8 ? T : sms * 8;
  noalloc_rows_kernel<<<grid, kThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(logits), ld, targets, T, V, ignore_index, smoothing,
      scratch, static_cast<__nv_bfloat16*>(dlogits));
  noalloc_reduce_kernel<<<1, 1024, 0, stream>>>(scratch, T, loss_out);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

// Capacity of the fixed scratch array, in rows.
extern "C" __attribute__((visibility("default"))) int flodl_softmax_ce_noalloc_max_rows() {
  return kNoAllocMaxRows;
}
