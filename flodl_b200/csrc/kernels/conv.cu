// Convolution and batch-norm building blocks for sm_100a (NHWC bf16 activations).
//
// Reference ops: at::conv2d / at::batch_norm / relu as called by floDl's
// Conv2d, BatchNorm2d and the ResNet-20 benchmark model
// (flodl-sys/ops_nn.cpp conv/batch_norm entry points, ddp-bench/src/models/resnet.rs).
//
// A convolution runs as an explicit column gather feeding the tcgen05 GEMM:
//   forward  cols[M, K] = im2col(x),   y[M, Cout]  = cols . Wp^T
//   dgrad    dcols[M, K] = dy . Wp,    dx = col2im(dcols) (+ skip gradient, x ReLU mask)
//   wgrad    dWp[Cout, K] += dy^T . cols                               (split-K f32)
// M = N*Ho*Wo output pixels, K = k*k*C with the column index (kh*k + kw)*C + ci:
// a tap's C channels are contiguous in both the NHWC activation and the
// column row, so the gather and scatter move 16-byte vectors (C is a multiple
// of 8; the 3-channel network input is zero-padded to 8). Wp is the weight
// packed in that order (bf16, from the f32 OIHW parameter) and dWp is unpacked
// back into the OIHW gradient - one launch each for all convolutions of a
// network (a table of layers).
//
// Batch norm (training) over the rows of a [M, C] bf16 matrix:
//   bn_stats      : per-channel sum / sum of squares -> mean, rstd; running-stat update
//   bn_apply      : y = relu?(gamma (x - mean) rstd + beta (+ identity))
//   bn_bwd_reduce : dz = dy (* [y > 0]); sums of dz and dz * xhat -> dgamma, dbeta
//   bn_bwd_apply  : dx = gamma rstd (dz - sum(dz)/M - xhat sum(dz xhat)/M) (and dz itself)
// The reductions finish in the kernel: every block adds its partials into a
// workspace with atomics, the last block to arrive (ticket counter) computes
// the per-channel results and resets the workspace for the next call.
#include "sm100_ptx.cuh"
#include "kernels.h"

namespace flodl {

namespace {

constexpr int kRedThreads = 256;

// Launch with programmatic dependent launch (every kernel of this file starts
// with pdl_wait, so it reads nothing before the previous kernel finished);
// returns from the calling launcher on a launch error.
#define FL_PDL(...)                                      \
  do {                                                   \
    const cudaError_t e_ = launch_pdl(__VA_ARGS__);      \
    if (e_ != cudaSuccess) return e_;                    \
  } while (0)

int blocks_for(int64_t work, int threads, int per_sm) {
  int64_t b = (work + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * per_sm;
  return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

// ---------------------------------------------------------------- im2col / col2im
// cols[pix, (kh*kw_ + kw)*C + c] = x[n, ho*sh - ph + kh, wo*sw - pw + kw, c] (0
// outside), for a kh_ x kw_ kernel with per-axis stride and padding.
// Thread = (output pixel, tap, group of 8 channels): one 16-byte load or zero,
// one 16-byte store.
__global__ void im2col_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ cols,
                              int N, int H, int W, int C, int Ho, int Wo, ConvGeo g2, uint32_t total,
                              FastDiv fG, FastDiv fKK, FastDiv fWo, FastDiv fHo, FastDiv fKw) {
  pdl_wait();
  pdl_trigger();
  const int kk = g2.kh * g2.kw;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t t = fG.div(i);
    const int g = (int)(i - t * fG.d);
    const uint32_t pix = fKK.div(t);
    const int tap = (int)(t - pix * kk);
    const uint32_t t2 = fWo.div(pix);
    const int wo = (int)(pix - t2 * Wo);
    const uint32_t n = fHo.div(t2);
    const int ho = (int)(t2 - n * Ho);
    const int tkh = (int)fKw.div(tap);
    const int h = ho * g2.sh - g2.ph + tkh;
    const int w = wo * g2.sw - g2.pw + (tap - tkh * g2.kw);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (h >= 0 && h < H && w >= 0 && w < W)
      v = *reinterpret_cast<const uint4*>(x + (((int64_t)n * H + h) * W + w) * C + g * 8);
    *reinterpret_cast<uint4*>(cols + (int64_t)pix * ((int64_t)kk * C) + tap * C + g * 8) = v;
  }
}

// Weight packing for all convolutions of a network in one launch:
//   packed[co, (kh*k + kw)*Cp + ci] = bf16(w[co, ci, kh, kw])   (0 for ci >= Cin)
// and the reverse for gradients:
//   grad[co, ci, kh, kw] += gacc[co, (kh*k + kw)*Cp + ci];  gacc <- 0
__global__ void pack_conv_weights_kernel(const ConvPackEntry* __restrict__ tab, int n) {
  pdl_wait();
  pdl_trigger();
  for (int e = blockIdx.y; e < n; e += gridDim.y) {
    const ConvPackEntry t = tab[e];
    const int K = t.k * t.k * t.cin_pad;
    const int total = t.cout * K;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
      const int co = i / K, r = i % K;
      const int tap = r / t.cin_pad, ci = r % t.cin_pad;
      const float v = ci < t.cin ? t.w[((size_t)co * t.cin + ci) * t.k * t.k + tap] : 0.f;
      t.packed[i] = __float2bfloat16_rn(v);
    }
  }
}

__global__ void unpack_conv_grads_kernel(const ConvPackEntry* __restrict__ tab, int n) {
  pdl_wait();
  pdl_trigger();
  for (int e = blockIdx.y; e < n; e += gridDim.y) {
    const ConvPackEntry t = tab[e];
    const int K = t.k * t.k * t.cin_pad;
    const int total = t.cout * K;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
      const int co = i / K, r = i % K;
      const int tap = r / t.cin_pad, ci = r % t.cin_pad;
      const float g = t.gacc[i];
      t.gacc[i] = 0.f;
      if (ci < t.cin) t.grad[((size_t)co * t.cin + ci) * t.k * t.k + tap] += g;
    }
  }
}

// ---------------------------------------------------------------- batch norm
// Shared shape of the reductions: thread = (row lane, channel group of 8);
// C/8 groups per row (C a multiple of 8, C <= 1024).
struct RowGroups {
  int groups, lanes, g, lane;
  __device__ RowGroups(int C) {
    groups = C / 8;
    lanes = kRedThreads / groups;
    g = threadIdx.x % groups;
    lane = threadIdx.x / groups;
  }
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = unpack_bf16x2(w[q]);
    v[2 * q] = f.x;
    v[2 * q + 1] = f.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Block-reduce two 8-wide accumulators of every (lane, group) over the lanes
// and add them into ws[0:C] / ws[C:2C]; returns true in every thread of the
// last block to finish (after which ws holds the grid totals).
__device__ bool reduce_into_workspace(const RowGroups& rg, int C, float (&a)[8], float (&b)[8],
                                      float* ws, unsigned* ticket) {
  __shared__ float red[kRedThreads / 32][32][17];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool pow2 = rg.groups <= 32 && (rg.groups & (rg.groups - 1)) == 0;
  if (pow2) {
    // threads of a warp with the same channel group differ in the bits above
    // log2(groups): butterfly over those, then one partial per warp and group
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      if (off < rg.groups) break;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        a[e] += __shfl_xor_sync(0xffffffffu, a[e], off);
        b[e] += __shfl_xor_sync(0xffffffffu, b[e], off);
      }
    }
    if (lane < rg.groups) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        red[warp][lane][e] = a[e];
        red[warp][lane][8 + e] = b[e];
      }
    }
    __syncthreads();
    if ((int)threadIdx.x < rg.groups) {
      float sa[8], sb[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) sa[e] = sb[e] = 0.f;
#pragma unroll
      for (int w = 0; w < kRedThreads / 32; ++w)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          sa[e] += red[w][threadIdx.x][e];
          sb[e] += red[w][threadIdx.x][8 + e];
        }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        atomicAdd(ws + threadIdx.x * 8 + e, sa[e]);
        atomicAdd(ws + C + threadIdx.x * 8 + e, sb[e]);
      }
    }
  } else {
    // general channel counts: lane-0 thread of each group sums over the lanes
    float* flat = &red[0][0][0];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      flat[threadIdx.x * 17 + e] = a[e];
      flat[threadIdx.x * 17 + 8 + e] = b[e];
    }
    __syncthreads();
    if (rg.lane == 0 && rg.g < rg.groups) {
      float sa[8], sb[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) sa[e] = sb[e] = 0.f;
      for (int l = 0; l < rg.lanes; ++l) {
        const int t = l * rg.groups + rg.g;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          sa[e] += flat[t * 17 + e];
          sb[e] += flat[t * 17 + 8 + e];
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        atomicAdd(ws + rg.g * 8 + e, sa[e]);
        atomicAdd(ws + C + rg.g * 8 + e, sb[e]);
      }
    }
  }
  __threadfence();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (last) __threadfence();
  return last;
}

// Last block of a batch-norm backward reduction: ws[0:2C] holds the grid's
// sum(dz) / sum(dz * xhat); keep them in out2 for the apply pass, accumulate
// dbeta / dgamma and leave ws and the ticket zeroed for the next call.
__device__ void bn_bwd_finish(int C, float* ws, float* out2, float* dgamma, float* dbeta,
                              unsigned* ticket) {
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float a = __ldcg(ws + c), b = __ldcg(ws + C + c);
    out2[c] = a;
    out2[C + c] = b;
    if (dbeta) dbeta[c] += a;
    if (dgamma) dgamma[c] += b;
    ws[c] = 0.f;
    ws[C + c] = 0.f;
  }
  if (threadIdx.x == 0) *ticket = 0u;
}

// dx[n, h, w, c] = sum over taps (kh, kw) whose output pixel (ho, wo) reads
// (h, w) of dcols[pix(ho, wo), (kh*k + kw)*C + c]; then + add[...] and, with a
// mask tensor, * [mask > 0] (the ReLU that produced the input). Thread =
// (input pixel, group of 8 channels).
template <typename TAdd, bool kBn>
__global__ void __launch_bounds__(256, kBn ? 4 : 1) col2im_kernel(
    const __nv_bfloat16* __restrict__ dcols, int ldc, __nv_bfloat16* __restrict__ dx,
    const TAdd* __restrict__ add, const __nv_bfloat16* __restrict__ mask, int N, int H, int W,
    int C, int Ho, int Wo, ConvGeo g2, BnBwdSums bn, uint32_t total, FastDiv fG, FastDiv fW,
    FastDiv fH, FastDiv fSh, FastDiv fSw) {
  pdl_wait();
  pdl_trigger();
  const int G = C / 8;
  const uint32_t stride = gridDim.x * blockDim.x;
  // with kBn the block size is a multiple of G, so a thread keeps its channel
  // group (threadIdx.x % G) on every iteration and sums it in registers; the
  // batch norm's mean / rstd wait in shared memory (C <= 2048), not registers
  float sd[8], sdx[8];
  __shared__ float4 s_mr[kBn ? 2 * 2048 / 4 : 1];
  if constexpr (kBn) {
    for (int c = threadIdx.x; c < C / 4; c += blockDim.x) {
      s_mr[c] = reinterpret_cast<const float4*>(bn.mean)[c];
      s_mr[512 + c] = reinterpret_cast<const float4*>(bn.rstd)[c];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) sd[e] = sdx[e] = 0.f;
    __syncthreads();
  }
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t pix = fG.div(i);
    const int g = (int)(i - pix * G);
    const uint32_t t = fW.div(pix);
    const int w = (int)(pix - t * W);
    const uint32_t n32 = fH.div(t);
    const int h = (int)(t - n32 * H);
    const int n = (int)n32;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int kh = 0; kh < g2.kh; ++kh) {
      const int hn = h + g2.ph - kh;
      if (hn < 0) continue;
      const int ho = (int)fSh.div((uint32_t)hn);
      if (ho * g2.sh != hn || ho >= Ho) continue;
      for (int kw = 0; kw < g2.kw; ++kw) {
        const int wn = w + g2.pw - kw;
        if (wn < 0) continue;
        const int wo = (int)fSw.div((uint32_t)wn);
        if (wo * g2.sw != wn || wo >= Wo) continue;
        const int64_t op = ((int64_t)n * Ho + ho) * Wo + wo;
        const uint4 u =
            *reinterpret_cast<const uint4*>(dcols + op * ldc + (kh * g2.kw + kw) * C + g * 8);
        const uint32_t ws[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(ws[q]);
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      }
    }
    const int64_t o = (int64_t)pix * C + g * 8;
    if (add) {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += to_f32(add[o + e]);
    }
    if (mask) {
      const uint4 u = *reinterpret_cast<const uint4*>(mask + o);
      const uint32_t ws[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(ws[q]);
        if (!(f.x > 0.f)) acc[2 * q] = 0.f;
        if (!(f.y > 0.f)) acc[2 * q + 1] = 0.f;
      }
    }
    uint4 out;
    out.x = pack_bf16x2(acc[0], acc[1]);
    out.y = pack_bf16x2(acc[2], acc[3]);
    out.z = pack_bf16x2(acc[4], acc[5]);
    out.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(dx + o) = out;
    if constexpr (kBn) {
      // sums of the stored (bf16) gradient, the values the apply pass reads
      float v[8], q[8];
      load8(bn.x + o, v);
      const uint32_t ow[4] = {out.x, out.y, out.z, out.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(ow[k]);
        q[2 * k] = f.x;
        q[2 * k + 1] = f.y;
      }
      const float4 m0 = s_mr[g * 2], m1 = s_mr[g * 2 + 1];
      const float4 r0 = s_mr[512 + g * 2], r1 = s_mr[512 + g * 2 + 1];
      const float mu[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
      const float rs[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        sd[e] += q[e];
        sdx[e] = fmaf(q[e], (v[e] - mu[e]) * rs[e], sdx[e]);
      }
    }
  }
  if constexpr (kBn) {
    RowGroups rg(C);
    if (!reduce_into_workspace(rg, C, sd, sdx, bn.ws, bn.ticket)) return;
    bn_bwd_finish(C, bn.ws, bn.sums, bn.dgamma, bn.dbeta, bn.ticket);
  }
}

__global__ void __launch_bounds__(kRedThreads) bn_stats_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t M, int C, float eps, float momentum,
    float* __restrict__ mean, float* __restrict__ rstd, float* __restrict__ run_mean,
    float* __restrict__ run_var, float* __restrict__ ws, unsigned* __restrict__ ticket) {
  pdl_wait();
  pdl_trigger();
  RowGroups rg(C);
  float s1[8], s2[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) s1[e] = s2[e] = 0.f;
  if (rg.lane < rg.lanes) {
#pragma unroll 4
    for (int64_t r = blockIdx.x * (int64_t)rg.lanes + rg.lane; r < M;
         r += (int64_t)gridDim.x * rg.lanes) {
      float v[8];
      load8(x + r * C + rg.g * 8, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s1[e] += v[e];
        s2[e] = fmaf(v[e], v[e], s2[e]);
      }
    }
  }
  if (!reduce_into_workspace(rg, C, s1, s2, ws, ticket)) return;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float mu = __ldcg(ws + c) / (float)M;
    const float var = fmaxf(__ldcg(ws + C + c) / (float)M - mu * mu, 0.f);
    mean[c] = mu;
    rstd[c] = rsqrtf(var + eps);
    if (run_mean) {
      const float unbiased = M > 1 ? var * (float)M / (float)(M - 1) : var;
      run_mean[c] = (1.f - momentum) * run_mean[c] + momentum * mu;
      run_var[c] = (1.f - momentum) * run_var[c] + momentum * unbiased;
    }
    ws[c] = 0.f;
    ws[C + c] = 0.f;
  }
  if (threadIdx.x == 0) *ticket = 0u;
}

__global__ void bn_apply_kernel(const __nv_bfloat16* __restrict__ x, int64_t M, int C,
                                const float* __restrict__ mean, const float* __restrict__ rstd,
                                const float* __restrict__ gamma, const float* __restrict__ beta,
                                const __nv_bfloat16* __restrict__ identity, int relu,
                                __nv_bfloat16* __restrict__ y, FastDiv fGroups) {
  pdl_wait();
  pdl_trigger();
  const uint32_t total = (uint32_t)M * fGroups.d;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t r32 = fGroups.div(i);
    const int c0 = (int)(i - r32 * fGroups.d) * 8;
    const int64_t r = r32;
    float v[8];
    load8(x + r * C + c0, v);
    float id[8];
    if (identity) load8(identity + r * C + c0, id);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int c = c0 + e;
      float o = (v[e] - __ldg(mean + c)) * __ldg(rstd + c);
      o = gamma ? fmaf(o, __ldg(gamma + c), beta ? __ldg(beta + c) : 0.f) : o;
      if (identity) o += id[e];
      v[e] = relu ? fmaxf(o, 0.f) : o;
    }
    store8(y + r * C + c0, v);
  }
}

// Batch norm applied from statistics a GEMM epilogue accumulated: ws[0:C]
// holds sum(y), ws[C:2C] sum(y^2) over the M rows. Every block derives mean
// and rstd for the channels (C <= kMaxBnC) in shared memory, block 0 writes
// them out and updates the running statistics, and the last block to finish
// re-zeroes the sums and the ticket for the next use.
constexpr int kMaxBnC = 1024;
__global__ void bn_apply_sums_kernel(const __nv_bfloat16* __restrict__ x, int64_t M, int C,
                                     float* __restrict__ ws, unsigned* __restrict__ ticket,
                                     float eps, float momentum, float* __restrict__ mean_out,
                                     float* __restrict__ rstd_out, float* __restrict__ run_mean,
                                     float* __restrict__ run_var,
                                     const float* __restrict__ gamma,
                                     const float* __restrict__ beta,
                                     const __nv_bfloat16* __restrict__ identity, int relu,
                                     __nv_bfloat16* __restrict__ y, FastDiv fGroups) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sc[kMaxBnC], sh[kMaxBnC];
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float mu = __ldcg(ws + c) / (float)M;
    const float var = fmaxf(__ldcg(ws + C + c) / (float)M - mu * mu, 0.f);
    const float rs = rsqrtf(var + eps);
    const float g = gamma ? gamma[c] : 1.f;
    sc[c] = rs * g;
    sh[c] = (beta ? beta[c] : 0.f) - mu * rs * g;
    if (blockIdx.x == 0) {
      mean_out[c] = mu;
      rstd_out[c] = rs;
      if (run_mean) {
        const float unbiased = M > 1 ? var * (float)M / (float)(M - 1) : var;
        run_mean[c] = (1.f - momentum) * run_mean[c] + momentum * mu;
        run_var[c] = (1.f - momentum) * run_var[c] + momentum * unbiased;
      }
    }
  }
  __syncthreads();
  const uint32_t total = (uint32_t)M * fGroups.d;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t r32 = fGroups.div(i);
    const int c0 = (int)(i - r32 * fGroups.d) * 8;
    const int64_t r = r32;
    float v[8];
    load8(x + r * C + c0, v);
    float id[8];
    if (identity) load8(identity + r * C + c0, id);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float o = fmaf(v[e], sc[c0 + e], sh[c0 + e]);
      if (identity) o += id[e];
      v[e] = relu ? fmaxf(o, 0.f) : o;
    }
    store8(y + r * C + c0, v);
  }
  // every block read the sums at its start; the last one to get here clears them
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last) {
    for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) ws[c] = 0.f;
    if (threadIdx.x == 0) *ticket = 0u;
  }
}

// sums of dz and dz * xhat per channel; the last block also accumulates
// dgamma += sum(dz xhat), dbeta += sum(dz) and keeps both sums in out2[0:2C]
__global__ void __launch_bounds__(kRedThreads) bn_bwd_reduce_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ ymask,
    const __nv_bfloat16* __restrict__ x, int64_t M, int C, const float* __restrict__ mean,
    const float* __restrict__ rstd, float* __restrict__ dgamma, float* __restrict__ dbeta,
    float* __restrict__ out2, float* __restrict__ ws, unsigned* __restrict__ ticket) {
  pdl_wait();
  pdl_trigger();
  RowGroups rg(C);
  float sd[8], sdx[8], mu[8], rs[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    sd[e] = sdx[e] = 0.f;
    mu[e] = rg.g < rg.groups ? __ldg(mean + rg.g * 8 + e) : 0.f;
    rs[e] = rg.g < rg.groups ? __ldg(rstd + rg.g * 8 + e) : 0.f;
  }
  if (rg.lane < rg.lanes) {
#pragma unroll 4
    for (int64_t r = blockIdx.x * (int64_t)rg.lanes + rg.lane; r < M;
         r += (int64_t)gridDim.x * rg.lanes) {
      float g[8], v[8];
      load8(dy + r * C + rg.g * 8, g);
      load8(x + r * C + rg.g * 8, v);
      if (ymask) {
        float m[8];
        load8(ymask + r * C + rg.g * 8, m);
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = m[e] > 0.f ? g[e] : 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        sd[e] += g[e];
        sdx[e] = fmaf(g[e], (v[e] - mu[e]) * rs[e], sdx[e]);
      }
    }
  }
  if (!reduce_into_workspace(rg, C, sd, sdx, ws, ticket)) return;
  bn_bwd_finish(C, ws, out2, dgamma, dbeta, ticket);
}

__global__ void bn_bwd_apply_kernel(const __nv_bfloat16* __restrict__ dy,
                                    const __nv_bfloat16* __restrict__ ymask,
                                    const __nv_bfloat16* __restrict__ x, int64_t M, int C,
                                    const float* __restrict__ mean, const float* __restrict__ rstd,
                                    const float* __restrict__ gamma, const float* __restrict__ sums,
                                    __nv_bfloat16* __restrict__ dx, __nv_bfloat16* __restrict__ dz_out,
                                    FastDiv fGroups) {
  pdl_wait();
  pdl_trigger();
  const uint32_t total = (uint32_t)M * fGroups.d;
  const float invM = 1.f / (float)M;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t r32 = fGroups.div(i);
    const int c0 = (int)(i - r32 * fGroups.d) * 8;
    const int64_t r = r32;
    float g[8], v[8];
    load8(dy + r * C + c0, g);
    load8(x + r * C + c0, v);
    if (ymask) {
      float m[8];
      load8(ymask + r * C + c0, m);
#pragma unroll
      for (int e = 0; e < 8; ++e) g[e] = m[e] > 0.f ? g[e] : 0.f;
    }
    if (dz_out) store8(dz_out + r * C + c0, g);
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int c = c0 + e;
      const float rsd = __ldg(rstd + c);
      const float xh = (v[e] - __ldg(mean + c)) * rsd;
      const float gm = gamma ? __ldg(gamma + c) : 1.f;
      o[e] = gm * rsd * (g[e] - __ldg(sums + c) * invM - xh * __ldg(sums + C + c) * invM);
    }
    store8(dx + r * C + c0, o);
  }
}

// ---------------------------------------------------------------- pooling
// y[n, c] = mean over the HW pixels of x[n, :, c]   (x NHWC bf16, y bf16)
__global__ void avgpool_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                   int N, int HW, int C) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = (int64_t)N * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const int n = (int)(i / C);
    float s = 0.f;
    for (int p = 0; p < HW; ++p) s += __bfloat162float(x[((int64_t)n * HW + p) * C + c]);
    y[i] = __float2bfloat16_rn(s / (float)HW);
  }
}

// dx[n, p, c] = dy[n, c] / HW   (dy with row pitch ld)
__global__ void avgpool_bwd_kernel(const __nv_bfloat16* __restrict__ dy, int ld,
                                   __nv_bfloat16* __restrict__ dx, int N, int HW, int C) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = (int64_t)N * HW * C;
  const float inv = 1.f / (float)HW;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const int n = (int)(i / ((int64_t)HW * C));
    dx[i] = __float2bfloat16_rn(__bfloat162float(dy[(int64_t)n * ld + c]) * inv);
  }
}

// NCHW f32 -> NHWC bf16 with Cp >= C channels (channels C..Cp-1 zero)
__global__ void nchw_to_nhwc_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                    int N, int C, int HW, int Cp) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = (int64_t)N * Cp * HW;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % Cp);
    const int64_t t = i / Cp;
    const int p = (int)(t % HW);
    const int n = (int)(t / HW);
    y[i] = __float2bfloat16_rn(c < C ? x[((int64_t)n * C + c) * HW + p] : 0.f);
  }
}

// bf16 copy of an f32 [rows, cols] matrix into a [rows, ld] buffer, zero-padding columns cols..ld-1
__global__ void cast_pad_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int rows,
                                int cols, int ld) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = (int64_t)rows * ld;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % ld);
    const int64_t r = i / ld;
    y[i] = __float2bfloat16_rn(c < cols ? x[r * cols + c] : 0.f);
  }
}

}  // namespace

static bool geo_ok(const ConvGeo& g) {
  return g.kh > 0 && g.kw > 0 && g.sh > 0 && g.sw > 0 && g.ph >= 0 && g.pw >= 0;
}

cudaError_t launch_im2col_geo(const __nv_bfloat16* x, __nv_bfloat16* cols, int N, int H, int W,
                              int C, const ConvGeo& g, cudaStream_t st) {
  if (!geo_ok(g)) return cudaErrorInvalidValue;
  const int Ho = (H + 2 * g.ph - g.kh) / g.sh + 1, Wo = (W + 2 * g.pw - g.kw) / g.sw + 1;
  if (Ho <= 0 || Wo <= 0 || C % 8) return cudaErrorInvalidValue;
  const int64_t total = (int64_t)N * Ho * Wo * g.kh * g.kw * (C / 8);
  if (total >= kMaxFlatIndex) return cudaErrorInvalidValue;
  FL_PDL(im2col_kernel, dim3(blocks_for(total, 256, 16)), dim3(256), 0, st, x, cols, N, H, W, C, Ho,
      Wo, g, (uint32_t)total, FastDiv(C / 8), FastDiv(g.kh * g.kw), FastDiv(Wo), FastDiv(Ho),
      FastDiv(g.kw));
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_col2im_geo(const __nv_bfloat16* dcols, int ldc, __nv_bfloat16* dx,
                              const void* add, bool add_f32, const __nv_bfloat16* mask, int N,
                              int H, int W, int C, const ConvGeo& g, cudaStream_t st,
                              const BnBwdSums* bn) {
  if (!geo_ok(g)) return cudaErrorInvalidValue;
  const int Ho = (H + 2 * g.ph - g.kh) / g.sh + 1, Wo = (W + 2 * g.pw - g.kw) / g.sw + 1;
  if (C % 8) return cudaErrorInvalidValue;
  const BnBwdSums none{};
  if (bn) {
    // the block keeps each thread on one channel group; a few blocks per SM
    // keep the per-block atomics into the 2C sums few
    if (!bn->x || !bn->mean || !bn->rstd || !bn->sums || !bn->ws || !bn->ticket ||
        256 % (C / 8) != 0 || (reinterpret_cast<uintptr_t>(bn->mean) & 15) ||
        (reinterpret_cast<uintptr_t>(bn->rstd) & 15))
      return cudaErrorInvalidValue;
  }
  const int64_t total64 = (int64_t)N * H * W * (C / 8);
  if (total64 >= kMaxFlatIndex) return cudaErrorInvalidValue;
  const uint32_t total = (uint32_t)total64;
  const FastDiv fG(C / 8), fW(W), fH(H), fSh(g.sh), fSw(g.sw);
  const int blocks = blocks_for(total64, 256, bn ? 4 : 16);
  const BnBwdSums& b = bn ? *bn : none;
  if (add_f32) {
    if (bn)
      FL_PDL(col2im_kernel<float, true>, dim3(blocks), dim3(256), 0, st, dcols, ldc, dx,
          (const float*)add, mask, N, H, W, C, Ho, Wo, g, b, total, fG, fW, fH, fSh, fSw);
    else
      FL_PDL(col2im_kernel<float, false>, dim3(blocks), dim3(256), 0, st, dcols, ldc, dx,
          (const float*)add, mask, N, H, W, C, Ho, Wo, g, b, total, fG, fW, fH, fSh, fSw);
  } else {
    const __nv_bfloat16* a16 = (const __nv_bfloat16*)add;
    if (bn)
      FL_PDL(col2im_kernel<__nv_bfloat16, true>, dim3(blocks), dim3(256), 0, st, dcols, ldc, dx,
          a16, mask, N, H, W, C, Ho, Wo, g, b, total, fG, fW, fH, fSh, fSw);
    else
      FL_PDL(col2im_kernel<__nv_bfloat16, false>, dim3(blocks), dim3(256), 0, st, dcols, ldc, dx,
          a16, mask, N, H, W, C, Ho, Wo, g, b, total, fG, fW, fH, fSh, fSw);
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_im2col(const __nv_bfloat16* x, __nv_bfloat16* cols, int N, int H, int W, int C,
                          int k, int s, int p, cudaStream_t st) {
  return launch_im2col_geo(x, cols, N, H, W, C, ConvGeo{k, k, s, s, p, p}, st);
}

cudaError_t launch_col2im(const __nv_bfloat16* dcols, int ldc, __nv_bfloat16* dx, const void* add,
                          bool add_f32, const __nv_bfloat16* mask, int N, int H, int W, int C,
                          int k, int s, int p, cudaStream_t st) {
  return launch_col2im_geo(dcols, ldc, dx, add, add_f32, mask, N, H, W, C, ConvGeo{k, k, s, s, p, p},
                           st);
}

cudaError_t launch_pack_conv_weights(const ConvPackEntry* table, int n, int max_elems,
                                     cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  dim3 grid((max_elems + 255) / 256, n);
  FL_PDL(pack_conv_weights_kernel, dim3(grid), dim3(256), 0, st, table, n);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_unpack_conv_grads(const ConvPackEntry* table, int n, int max_elems,
                                     cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  dim3 grid((max_elems + 255) / 256, n);
  FL_PDL(unpack_conv_grads_kernel, dim3(grid), dim3(256), 0, st, table, n);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_bn_stats(const __nv_bfloat16* x, int64_t M, int C, float eps, float momentum,
                            float* mean, float* rstd, float* run_mean, float* run_var, float* ws,
                            unsigned* ticket, cudaStream_t st) {
  if (C % 8 || C / 8 > kRedThreads) return cudaErrorInvalidValue;
  const int lanes = kRedThreads / (C / 8);
  FL_PDL(bn_stats_kernel, dim3(blocks_for((M + lanes - 1) / lanes, 4, 2)), dim3(kRedThreads), 0, st,
      x, M, C, eps, momentum, mean, rstd, run_mean, run_var, ws, ticket);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_bn_apply(const __nv_bfloat16* x, int64_t M, int C, const float* mean,
                            const float* rstd, const float* gamma, const float* beta,
                            const __nv_bfloat16* identity, bool relu, __nv_bfloat16* y,
                            cudaStream_t st) {
  if (C % 8 || M * (C / 8) >= kMaxFlatIndex) return cudaErrorInvalidValue;
  FL_PDL(bn_apply_kernel, dim3(blocks_for(M * (C / 8), 256, 16)), dim3(256), 0, st, x, M, C, mean,
      rstd, gamma, beta, identity, relu ? 1 : 0, y, FastDiv(C / 8));
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_bn_apply_sums(const __nv_bfloat16* x, int64_t M, int C, float* ws,
                                 unsigned* ticket, float eps, float momentum, float* mean,
                                 float* rstd, float* run_mean, float* run_var, const float* gamma,
                                 const float* beta, const __nv_bfloat16* identity, bool relu,
                                 __nv_bfloat16* y, cudaStream_t st) {
  if (C % 8 || C > kMaxBnC || M <= 0 || M * (C / 8) >= kMaxFlatIndex)
    return cudaErrorInvalidValue;
  FL_PDL(bn_apply_sums_kernel, dim3(blocks_for(M * (C / 8), 256, 16)), dim3(256), 0, st, x, M, C,
      ws, ticket, eps, momentum, mean, rstd, run_mean, run_var, gamma, beta, identity, relu ? 1 : 0,
      y, FastDiv(C / 8));
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_bn_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* ymask,
                          const __nv_bfloat16* x, int64_t M, int C, const float* mean,
                          const float* rstd, const float* gamma, float* dgamma, float* dbeta,
                          float* sums, float* ws, unsigned* ticket, __nv_bfloat16* dx,
                          __nv_bfloat16* dz_out, cudaStream_t st) {
  if (C % 8 || C / 8 > kRedThreads) return cudaErrorInvalidValue;
  const int lanes = kRedThreads / (C / 8);
  FL_PDL(bn_bwd_reduce_kernel, dim3(blocks_for((M + lanes - 1) / lanes, 4, 2)), dim3(kRedThreads),
      0, st, dy, ymask, x, M, C, mean, rstd, dgamma, dbeta, sums, ws, ticket);
  note_launch();
  return launch_bn_bwd_apply(dy, ymask, x, M, C, mean, rstd, gamma, sums, dx, dz_out, st);
}

cudaError_t launch_bn_bwd_apply(const __nv_bfloat16* dy, const __nv_bfloat16* ymask,
                                const __nv_bfloat16* x, int64_t M, int C, const float* mean,
                                const float* rstd, const float* gamma, const float* sums,
                                __nv_bfloat16* dx, __nv_bfloat16* dz_out, cudaStream_t st) {
  if (C % 8 || M * (C / 8) >= kMaxFlatIndex) return cudaErrorInvalidValue;
  FL_PDL(bn_bwd_apply_kernel, dim3(blocks_for(M * (C / 8), 256, 16)), dim3(256), 0, st, dy, ymask,
      x, M, C, mean, rstd, gamma, sums, dx, dz_out, FastDiv(C / 8));
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_avgpool_fwd(const __nv_bfloat16* x, __nv_bfloat16* y, int N, int HW, int C,
                               cudaStream_t st) {
  FL_PDL(avgpool_fwd_kernel, dim3(blocks_for((int64_t)N * C, 256, 4)), dim3(256), 0, st, x, y, N,
      HW, C);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_avgpool_bwd(const __nv_bfloat16* dy, int ld, __nv_bfloat16* dx, int N, int HW,
                               int C, cudaStream_t st) {
  FL_PDL(avgpool_bwd_kernel, dim3(blocks_for((int64_t)N * HW * C, 256, 16)), dim3(256), 0, st, dy,
      ld, dx, N, HW, C);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_nchw_to_nhwc(const float* x, __nv_bfloat16* y, int N, int C, int HW, int Cp,
                                cudaStream_t st) {
  FL_PDL(nchw_to_nhwc_kernel, dim3(blocks_for((int64_t)N * Cp * HW, 256, 16)), dim3(256), 0, st, x,
      y, N, C, HW, Cp);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_cast_pad(const float* x, __nv_bfloat16* y, int rows, int cols, int ld,
                            cudaStream_t st) {
  FL_PDL(cast_pad_kernel, dim3(blocks_for((int64_t)rows * ld, 256, 4)), dim3(256), 0, st, x, y,
      rows, cols, ld);
  note_launch();
  return cudaGetLastError();
}

}  // namespace flodl
