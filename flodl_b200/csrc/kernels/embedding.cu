// Fused token (+position, +token-type) embedding for sm_100a.
//
// Reference: at::embedding (flodl-sys/ops_training.cpp:1302-1330) followed by
// separate adds for positional/type tables in the model code. Here one pass
// gathers and sums the rows and writes the f32 residual stream (and optionally
// its bf16 copy). Backward: the token-table gradient goes through a one-hot
// tcgen05 GEMM for small vocabularies (no atomics contention) or vectorised
// atomics for large ones; the position gradient is a reduction over the batch.
#include "sm100_ptx.cuh"
#include "kernels.h"

namespace flodl {

namespace {

__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ tok,
                                 const float* __restrict__ pos, const int64_t* __restrict__ type_ids,
                                 const float* __restrict__ type_tab, float* __restrict__ out,
                                 __nv_bfloat16* __restrict__ out_bf16, int T, int S, int C, int V,
                                 FastDiv fC4, FastDiv fS) {
  pdl_wait();
  pdl_trigger();
  const uint32_t total = (uint32_t)T * fC4.d;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int t = (int)fC4.div(i);
    const int c = (int)(i - (uint32_t)t * fC4.d) * 4;
    int64_t id = ids[t];
    if (id < 0 || id >= V) id = 0;  // out-of-range ids read row 0 (checked on the host side)
    float4 v = *reinterpret_cast<const float4*>(tok + id * C + c);
    if (pos) {
      const int s = t - (int)fS.div((uint32_t)t) * S;
      float4 p = *reinterpret_cast<const float4*>(pos + (int64_t)s * C + c);
      v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
    }
    if (type_tab) {
      const int64_t ty = type_ids ? type_ids[t] : 0;
      float4 p = *reinterpret_cast<const float4*>(type_tab + ty * C + c);
      v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
    }
    if (out) *reinterpret_cast<float4*>(out + (int64_t)t * C + c) = v;
    if (out_bf16) {
      uint2 u;
      u.x = pack_bf16x2(v.x, v.y);
      u.y = pack_bf16x2(v.z, v.w);
      *reinterpret_cast<uint2*>(out_bf16 + (int64_t)t * C + c) = u;
    }
  }
}

__global__ void embed_bwd_atomic_kernel(const int64_t* __restrict__ ids, const float* __restrict__ dy,
                                        float* __restrict__ dtok, int T, int C) {
  const int C4 = C / 4;
  const int64_t total = (int64_t)T * C4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / C4);
    const int c = (int)(i % C4) * 4;
    const int64_t id = ids[t];
    float4 g = *reinterpret_cast<const float4*>(dy + (int64_t)t * C + c);
    red_add_v4(dtok + id * C + c, g.x, g.y, g.z, g.w);
  }
}

// dpos[s, c] += sum_b dy[b, s, c]; four independent partial sums keep four
// loads in flight per thread
__global__ void pos_grad_kernel(const float* __restrict__ dy, float* __restrict__ dpos, int B, int S,
                                int C) {
  const int64_t total = (int64_t)S * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    int b = 0;
    for (; b + 4 <= B; b += 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u) s[u] += __ldg(dy + (int64_t)(b + u) * total + i);
    }
    for (; b < B; ++b) s[0] += __ldg(dy + (int64_t)b * total + i);
    dpos[i] += (s[0] + s[1]) + (s[2] + s[3]);
  }
}

// one_hot[t, v] = (ids[t] == v), eight columns (one 16-byte store) per
// thread; V % 8 == 0 and T * V / 8 < 2^31 (checked by the launcher)
__global__ void onehot_kernel(const int64_t* __restrict__ ids, __nv_bfloat16* __restrict__ out,
                              int T, int V, FastDiv fV8) {
  const uint32_t total = (uint32_t)T * fV8.d;
  const uint32_t one = 0x3f80u;  // bf16 1.0
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t t = fV8.div(i);
    const int v0 = (int)(i - t * fV8.d) * 8;
    const int64_t id = __ldg(ids + t);
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      w[q] = (id == v0 + 2 * q ? one : 0u) | ((id == v0 + 2 * q + 1 ? one : 0u) << 16);
    reinterpret_cast<uint4*>(out)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void onehot_scalar_kernel(const int64_t* __restrict__ ids,
                                     __nv_bfloat16* __restrict__ out, int T, int V) {
  const int64_t total = (int64_t)T * V;
  const __nv_bfloat16 one = __float2bfloat16_rn(1.f), zero = __float2bfloat16_rn(0.f);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / V);
    out[i] = (ids[t] == (int)(i % V)) ? one : zero;
  }
}

int grid_1d(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * 16;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

}  // namespace

cudaError_t launch_embed_fwd(const int64_t* ids, const float* tok, const float* pos,
                             const int64_t* type_ids, const float* type_tab, float* out,
                             __nv_bfloat16* out_bf16, int T, int S, int C, int V, cudaStream_t st) {
  if (C % 4 || (pos && S <= 0) || (int64_t)T * (C / 4) >= kMaxFlatIndex)
    return cudaErrorInvalidValue;
  cudaError_t e = launch_pdl(embed_fwd_kernel, dim3(grid_1d((int64_t)T * C / 4, 256)), dim3(256),
                             0, st, ids, tok, pos, type_ids, type_tab, out, out_bf16, T, S, C, V,
                             FastDiv(C / 4), FastDiv(S > 0 ? S : 1));
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_embed_bwd_atomic(const int64_t* ids, const float* dy, float* dtok, int T, int C,
                                    cudaStream_t st) {
  if (C % 4) return cudaErrorInvalidValue;
  embed_bwd_atomic_kernel<<<grid_1d((int64_t)T * C / 4, 256), 256, 0, st>>>(ids, dy, dtok, T, C);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_pos_grad(const float* dy, float* dpos, int B, int S, int C, cudaStream_t st) {
  pos_grad_kernel<<<grid_1d((int64_t)S * C, 256), 256, 0, st>>>(dy, dpos, B, S, C);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_onehot_bf16(const int64_t* ids, __nv_bfloat16* out, int T, int V,
                               cudaStream_t st) {
  if (V % 8 || (int64_t)T * (V / 8) >= kMaxFlatIndex || (reinterpret_cast<uintptr_t>(out) & 15))
    onehot_scalar_kernel<<<grid_1d((int64_t)T * V, 256), 256, 0, st>>>(ids, out, T, V);
  else
    onehot_kernel<<<grid_1d((int64_t)T * V / 8, 256), 256, 0, st>>>(ids, out, T, V,
                                                                     FastDiv(V / 8));
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
