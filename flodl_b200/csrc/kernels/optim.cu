// Fused optimizer updates over flat parameter arenas (sm_100a, memory-bound).
//
// Reference: at::_fused_adamw_/_fused_adam_ multi-tensor kernels
// (flodl-sys/ops_training.cpp:795-884) and the foreach SGD-momentum path
// (flodl/src/nn/optim/sgd.rs). Parameters, gradients and moments here live in
// contiguous f32 arenas, so one launch updates a whole parameter group. The
// kernel also refreshes the bf16 shadow of the weights that the forward GEMMs
// read, applies an optional gradient scale (global-norm clip coefficient or
// 1/world_size), and can zero the gradient in the same pass.
//
// lr, step and the clip coefficient are read from device memory so a CUDA
// graph that captures the step replays correctly as they change.
#include "sm100_ptx.cuh"
#include "kernels.h"

namespace flodl {

namespace {

int grid_1d(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * 8;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

__device__ __forceinline__ void adamw_elem(float& p, float g, float& m, float& v, float lr,
                                           float b1, float b2, float eps, float wd, float bc1,
                                           float bc2_sqrt, bool decoupled) {
  if (!decoupled) g += wd * p;
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  const float denom = sqrtf(v) / bc2_sqrt + eps;
  if (decoupled) p *= (1.f - lr * wd);
  p -= (lr / bc1) * m / denom;
}

__global__ void __launch_bounds__(256) adamw_kernel(AdamWArgs a) {
  pdl_wait();
  pdl_trigger();
  const float lr = *a.lr;
  const float t = *a.step;
  const float bc1 = 1.f - powf(a.beta1, t);
  const float bc2_sqrt = sqrtf(1.f - powf(a.beta2, t));
  const float gs = a.gscale ? *a.gscale : 1.f;
  const int64_t n4 = a.n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 p = reinterpret_cast<float4*>(a.p)[i];
    float4 g = reinterpret_cast<const float4*>(a.g)[i];
    float4 m = reinterpret_cast<float4*>(a.m)[i];
    float4 v = reinterpret_cast<float4*>(a.v)[i];
    adamw_elem(p.x, g.x * gs, m.x, v.x, lr, a.beta1, a.beta2, a.eps, a.wd, bc1, bc2_sqrt, a.decoupled);
    adamw_elem(p.y, g.y * gs, m.y, v.y, lr, a.beta1, a.beta2, a.eps, a.wd, bc1, bc2_sqrt, a.decoupled);
    adamw_elem(p.z, g.z * gs, m.z, v.z, lr, a.beta1, a.beta2, a.eps, a.wd, bc1, bc2_sqrt, a.decoupled);
    adamw_elem(p.w, g.w * gs, m.w, v.w, lr, a.beta1, a.beta2, a.eps, a.wd, bc1, bc2_sqrt, a.decoupled);
    reinterpret_cast<float4*>(a.p)[i] = p;
    reinterpret_cast<float4*>(a.m)[i] = m;
    reinterpret_cast<float4*>(a.v)[i] = v;
    if (a.zero_grad) reinterpret_cast<float4*>(a.g)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.shadow) {
      uint2 u;
      u.x = pack_bf16x2(p.x, p.y);
      u.y = pack_bf16x2(p.z, p.w);
      reinterpret_cast<uint2*>(a.shadow)[i] = u;
    }
  }
  // tail
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < a.n; i += stride) {
    float p = a.p[i], m = a.m[i], v = a.v[i];
    adamw_elem(p, a.g[i] * gs, m, v, lr, a.beta1, a.beta2, a.eps, a.wd, bc1, bc2_sqrt, a.decoupled);
    a.p[i] = p;
    a.m[i] = m;
    a.v[i] = v;
    if (a.zero_grad) a.g[i] = 0.f;
    if (a.shadow) a.shadow[i] = __float2bfloat16_rn(p);
  }
}

__device__ __forceinline__ void sgd_elem(float& p, float g, float* buf, bool first, float lr,
                                         float mom, float damp, float wd, bool nesterov) {
  g += wd * p;
  if (buf) {
    float b = first ? g : mom * (*buf) + (1.f - damp) * g;
    *buf = b;
    g = nesterov ? g + mom * b : b;
  }
  p -= lr * g;
}

__global__ void __launch_bounds__(256) sgd_kernel(SgdArgs a) {
  const float lr = *a.lr;
  const float gs = a.gscale ? *a.gscale : 1.f;
  const bool first = a.first ? (*a.first != 0.f) : false;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < a.n; i += stride) {
    float p = a.p[i];
    sgd_elem(p, a.g[i] * gs, a.buf ? a.buf + i : nullptr, first, lr, a.momentum, a.dampening, a.wd,
             a.nesterov);
    a.p[i] = p;
    if (a.zero_grad) a.g[i] = 0.f;
    if (a.shadow) a.shadow[i] = __float2bfloat16_rn(p);
  }
}

__global__ void sumsq_kernel(const float* __restrict__ x, int64_t n, float* out) {
  float s = 0.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float v = x[i];
    s += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float sh[32];
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += sh[i];
    atomicAdd(out, t);
  }
}

__global__ void clip_coef_kernel(const float* sumsq, float max_norm, float* coef, float* norm) {
  const float nrm = sqrtf(*sumsq);
  if (norm) *norm = nrm;
  *coef = fminf(1.f, max_norm / (nrm + 1e-6f));
}

__global__ void add_scalar_kernel(float* x, float v) { *x += v; }

__global__ void cast_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = __float2bfloat16_rn(x[i]);
}

}  // namespace

cudaError_t launch_adamw(const AdamWArgs& a, cudaStream_t st) {
  if (a.n <= 0) return cudaSuccess;
  if ((reinterpret_cast<uintptr_t>(a.p) | reinterpret_cast<uintptr_t>(a.g) |
       reinterpret_cast<uintptr_t>(a.m) | reinterpret_cast<uintptr_t>(a.v)) & 15)
    return cudaErrorMisalignedAddress;
  if (a.shadow && (reinterpret_cast<uintptr_t>(a.shadow) & 7)) return cudaErrorMisalignedAddress;
  cudaError_t e = launch_pdl(adamw_kernel, dim3(grid_1d(a.n / 4 + 1, 256)), dim3(256), 0, st, a);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_sgd(const SgdArgs& a, cudaStream_t st) {
  if (a.n <= 0) return cudaSuccess;
  sgd_kernel<<<grid_1d(a.n, 256), 256, 0, st>>>(a);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_sumsq(const float* x, int64_t n, float* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  sumsq_kernel<<<grid_1d(n, 256), 256, 0, st>>>(x, n, out);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_clip_coef(const float* sumsq, float max_norm, float* coef, float* norm,
                             cudaStream_t st) {
  clip_coef_kernel<<<1, 1, 0, st>>>(sumsq, max_norm, coef, norm);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_add_scalar(float* x, float v, cudaStream_t st) {
  add_scalar_kernel<<<1, 1, 0, st>>>(x, v);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_cast_f32_bf16(const float* x, __nv_bfloat16* y, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  cast_kernel<<<grid_1d(n, 256), 256, 0, st>>>(x, y, n);
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
