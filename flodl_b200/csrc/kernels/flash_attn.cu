// Flash attention forward/backward for sm_100a on tcgen05 tensor cores.
//
// Reference op: at::scaled_dot_product_attention (flodl-sys/ops_nn.cpp:407-431),
// used by MultiheadAttention (flodl/src/nn/attention.rs:136-230).
//
// Layout: Q/K/V are read from the packed projection output qkv [B*S, 3*H*D]
// (head h of Q at column h*D, of K at C+h*D, of V at 2C+h*D, C = H*D) through
// 3-D TMA maps {cols, S, B}, so rows past S in a batch are zero-filled and no
// transpose runs around the kernel. O is written token-major [B*S, C].
// Head dim D = 64 (one 128-byte swizzle row).
//
// Forward, one CTA per (128 queries, head, batch), 192 threads:
//   warp 0: TMA (Q once, K/V double-buffered), warp 1: MMA issue,
//   warps 2-5: softmax (thread = query row).
//   S = Q K^T -> TMEM (128 cols); P (bf16) -> shared memory (128B swizzle);
//   O_j = P V_j -> TMEM (64 cols), folded into register accumulators with the
//   online-softmax correction. lse is stored in base 2: lse2 = m2 + log2(l).
//
// Backward, one CTA per (128 keys, head, batch), looping over query tiles:
//   S^T = K Q^T, dP^T = V dO^T            (TMEM)
//   P^T = exp2(S^T*scale*log2e - lse2), dS^T = P^T (dP^T - delta)   (thread = key)
//   dV += P^T dO, dK += dS^T Q            (TMEM accumulators)
//   dQ_i = dS K  -> f32 atomics into a dQ accumulator, converted at the end.
// All waits are bounded (see sm100_ptx.cuh).
#include "sm100_ptx.cuh"
#include "flash_attn.h"

#include <mutex>

namespace flodl {

namespace {

constexpr int kTile = 128;  // queries per fwd CTA, keys per bwd CTA, and the other tile dim
constexpr int kD = 64;
constexpr int kTileBytes = kTile * kD * 2;  // 16 KB: 128 rows x 128 B
constexpr float kLog2e = 1.4426950408889634f;

__device__ uint64_t g_fa_wait_limit_ns = 2000000000ull;
// Optional progress words (host-mapped, 8 per CTA: one per warp, code = stage).
// Null unless a diagnostic run sets it; only lane 0 of a warp writes.
__device__ uint32_t* g_fa_progress = nullptr;

__device__ __forceinline__ void progress(int code) {
  uint32_t* p = g_fa_progress;
  if (p != nullptr && (threadIdx.x & 31) == 0) {
    const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    volatile uint32_t* w = p + cta * 8 + (threadIdx.x >> 5);
    *w = (uint32_t)code;
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled is a driver call and needs a context current on the
// calling thread. A runtime-API thread gets one lazily on its first runtime
// call that needs it, so a fresh thread (e.g. an autograd device thread whose
// first CUDA work is this launch) may have none yet: CUDA_ERROR_INVALID_CONTEXT.
// cudaSetDevice makes the device's primary context current; done once per
// thread and device.
static void bind_current_context() {
  thread_local int bound = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  if (bound != dev) {
    cudaSetDevice(dev);
    bound = dev;
  }
}

EncodeTiledFn encode_fn() {
  bind_current_context();
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D bf16 map over a [B, S, cols] token-major buffer; box = 64 cols x 128 rows x 1.
bool make_map_3d(CUtensorMap* m, const void* base, int B, int S, int cols) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)S * cols * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)kTile, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
             es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Store 8 bf16 (one 16-byte chunk) of row r, chunk index `chunk` (0..7) of a
// 128-row x 128-byte SW128 K-major block.
__device__ __forceinline__ void st_sw128_chunk(uint8_t* blk, int r, int chunk, uint4 v) {
  const int phys = chunk ^ (r & 7);
  *reinterpret_cast<uint4*>(blk + r * 128 + phys * 16) = v;
}

// Write 32 consecutive bf16 values (columns c0..c0+31 of a 128-column tile
// stored as two 64-column SW128 blocks of 16 KB) for row r.
__device__ __forceinline__ void st_row32_sw128(uint8_t* tile, int r, int c0, const float* v) {
  uint8_t* blk = tile + (c0 / 64) * kTileBytes;
  const int cc0 = c0 % 64;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
    w.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
    w.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
    w.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
    st_sw128_chunk(blk, r, cc0 / 8 + q, w);
  }
}

// ============================================================== forward
struct FwdSmem {
  uint8_t q[kTileBytes];
  uint8_t k[2][kTileBytes];
  uint8_t v[2][kTileBytes];
  uint8_t p[2 * kTileBytes];  // P tile: 128 queries x 128 keys, two 64-key blocks
  uint64_t q_full;
  uint64_t kv_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full, s_free, p_full, o_full, drain;
  uint32_t tmem_base;
  uint32_t abort;
};

__global__ void __launch_bounds__(192, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, __nv_bfloat16* __restrict__ out,
                     float* __restrict__ lse2, const uint8_t* __restrict__ key_pad, int B, int S,
                     int H, int causal, float scale, uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  FwdSmem& sm = *reinterpret_cast<FwdSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kTile;
  const int C = H * kD;
  const int n_kv_total = (S + kTile - 1) / kTile;
  const int n_kv = causal ? min(qt + 1, n_kv_total) : n_kv_total;
  const uint64_t limit = g_fa_wait_limit_ns;
  volatile uint32_t* abort_flag = &sm.abort;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, 4);
    mbar_init(&sm.p_full, 4);
    mbar_init(&sm.o_full, 1);
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<256>(&sm.tmem_base);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t t_s = tmem;        // S: 128 columns
  const uint32_t t_o = tmem + 128;  // O_j: 64 columns

  if (warp == 0) {
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_qkv);
      mbar_arrive_expect_tx(&sm.q_full, kTileBytes);
      tma_load_3d(sm.q, &tm_qkv, &sm.q_full, h * kD, q0, b);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_bounded(&sm.kv_empty[st], ph ^ 1, abort_flag, err, limit)) break;
        mbar_arrive_expect_tx(&sm.kv_full[st], 2 * kTileBytes);
        tma_load_3d(sm.k[st], &tm_qkv, &sm.kv_full[st], C + h * kD, j * kTile, b);
        tma_load_3d(sm.v[st], &tm_qkv, &sm.kv_full[st], 2 * C + h * kD, j * kTile, b);
      }
    }
    __syncwarp();  // reconverge the warp before the CTA-wide barrier below
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(128, kD, 0, 1);
      const uint32_t q_addr = smem_u32(sm.q);
      const uint32_t p_addr = smem_u32(sm.p);
      bool ok = mbar_wait_bounded(&sm.q_full, 0, abort_flag, err, limit);
      auto issue_s = [&](int j) {
        const int st = j & 1;
        const uint32_t k_addr = smem_u32(sm.k[st]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          umma_bf16(t_s, make_sdesc_sw128(q_addr + kk * 32, 16, 1024),
                    make_sdesc_sw128(k_addr + kk * 32, 16, 1024), idesc_s, kk > 0);
        umma_commit(&sm.s_full);
      };
      if (ok) ok = mbar_wait_bounded(&sm.kv_full[0], 0, abort_flag, err, limit);
      if (ok) issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv) {
          const int st1 = (j + 1) & 1;
          ok = mbar_wait_bounded(&sm.kv_full[st1], ((j + 1) >> 1) & 1, abort_flag, err, limit) &&
               mbar_wait_bounded(&sm.s_free, j & 1, abort_flag, err, limit);
          if (!ok) break;
          tc_fence_after();
          issue_s(j + 1);
        }
        ok = mbar_wait_bounded(&sm.p_full, j & 1, abort_flag, err, limit);
        if (!ok) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm.v[j & 1]);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint64_t a = make_sdesc_sw128(p_addr + (kk / 4) * kTileBytes + (kk % 4) * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(v_addr + kk * 2048, kTileBytes, 1024);
          umma_bf16(t_o, a, bd, idesc_o, kk > 0);
        }
        umma_commit(&sm.o_full);
        umma_commit(&sm.kv_empty[j & 1]);
      }
      if (!ok) {
        umma_commit(&sm.drain);
        uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&sm.drain, 0) && global_timer_ns() - t0 < 100000000ull) {
        }
      }
    }
    __syncwarp();  // reconverge the warp before the CTA-wide barrier below
  } else {
    // --------------------------------------------------- softmax warps
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // query row within the tile
    const int qi = q0 + r;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float sl2 = scale * kLog2e;
    float m_run = -INFINITY, l_run = 0.f, corr_prev = 0.f;
    float o_acc[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) o_acc[d] = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = mbar_wait_bounded(&sm.s_full, j & 1, abort_flag, err, limit);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      float s[kTile];
#pragma unroll
      for (int c = 0; c < kTile / 32; ++c) {
        uint32_t raw[32];
        tmem_ld_32cols(t_s + lane_off + c * 32, raw);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(raw[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free);
      // scale + mask
      const int k0 = j * kTile;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kTile; ++c) {
        const int kj = k0 + c;
        bool valid = kj < S && (!causal || kj <= qi);
        if (key_pad && kj < S) valid = valid && (key_pad[(size_t)b * S + kj] == 0);
        s[c] = valid ? s[c] * sl2 : -INFINITY;
        mx = fmaxf(mx, s[c]);
      }
      const float m_new = fmaxf(m_run, mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float corr = (m_run == -INFINITY) ? 0.f : exp2f(m_run - m_use);
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < kTile; ++c) {
        s[c] = exp2f(s[c] - m_use);
        rs += s[c];
      }
      l_run = l_run * corr + rs;
      m_run = m_new;
      // fold O_{j-1} (computed with the previous max) into the accumulator
      if (j > 0) {
        ok = mbar_wait_bounded(&sm.o_full, (j - 1) & 1, abort_flag, err, limit);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t raw[32];
          tmem_ld_32cols(t_o + lane_off + c * 32, raw);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            o_acc[c * 32 + i] = o_acc[c * 32 + i] * corr_prev + __uint_as_float(raw[i]);
        }
      }
      corr_prev = corr;
      // P -> shared memory (bf16, SW128 K-major), then hand it to the MMA warp
#pragma unroll
      for (int c = 0; c < kTile; c += 32) st_row32_sw128(sm.p, r, c, &s[c]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full);
    }
    if (ok) {
      ok = mbar_wait_bounded(&sm.o_full, (n_kv - 1) & 1, abort_flag, err, limit);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t raw[32];
        tmem_ld_32cols(t_o + lane_off + c * 32, raw);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          o_acc[c * 32 + i] = o_acc[c * 32 + i] * corr_prev + __uint_as_float(raw[i]);
      }
      if (qi < S) {
        const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
        __nv_bfloat16* orow = out + ((size_t)b * S + qi) * C + h * kD;
#pragma unroll
        for (int q = 0; q < kD / 8; ++q) {
          uint4 w;
          w.x = pack_bf16x2(o_acc[8 * q + 0] * inv_l, o_acc[8 * q + 1] * inv_l);
          w.y = pack_bf16x2(o_acc[8 * q + 2] * inv_l, o_acc[8 * q + 3] * inv_l);
          w.z = pack_bf16x2(o_acc[8 * q + 4] * inv_l, o_acc[8 * q + 5] * inv_l);
          w.w = pack_bf16x2(o_acc[8 * q + 6] * inv_l, o_acc[8 * q + 7] * inv_l);
          reinterpret_cast<uint4*>(orow)[q] = w;
        }
        lse2[((size_t)b * H + h) * S + qi] =
            (l_run > 0.f) ? (m_run + log2f(l_run)) : -INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<256>(tmem);
  }
}

// ============================================================== backward
struct BwdSmem {
  uint8_t k[kTileBytes];
  uint8_t v[kTileBytes];
  uint8_t q[2][kTileBytes];
  uint8_t dout[2][kTileBytes];
  uint8_t p[2 * kTileBytes];   // P^T: 128 keys x 128 queries
  uint8_t ds[2 * kTileBytes];  // dS^T: 128 keys x 128 queries
  uint64_t kv_full;
  uint64_t qdo_full[2];
  uint64_t qdo_empty[2];
  uint64_t sdp_full, pds_ready, dq_full, dq_free, drain;
  uint32_t tmem_base;
  uint32_t abort;
};

// delta[b,h,s] = sum_d dO * O ; also zeroes the f32 dQ accumulator rows.
__global__ void flash_bwd_pre_kernel(const __nv_bfloat16* __restrict__ dout,
                                     const __nv_bfloat16* __restrict__ out, float* __restrict__ delta,
                                     float* __restrict__ dq_acc, int B, int S, int H) {
  const int C = H * kD;
  const int64_t rows = (int64_t)B * S * H;
  const int warp_g = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * blockDim.x / 32;
  for (int64_t rw = warp_g; rw < rows; rw += nw) {
    const int64_t tok = rw / H;
    const int h = (int)(rw % H);
    const __nv_bfloat16* a = dout + tok * C + h * kD;
    const __nv_bfloat16* o = out + tok * C + h * kD;
    float2 x = unpack_bf16x2(reinterpret_cast<const uint32_t*>(a)[lane]);
    float2 y = unpack_bf16x2(reinterpret_cast<const uint32_t*>(o)[lane]);
    float s = x.x * y.x + x.y * y.y;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    const int b = (int)(tok / S), si = (int)(tok % S);
    if (lane == 0) delta[((int64_t)b * H + h) * S + si] = s;
    float2* dq = reinterpret_cast<float2*>(dq_acc + tok * C + h * kD);
    dq[lane] = make_float2(0.f, 0.f);
  }
}

// dqkv[:, q cols] = bf16(dq_acc * scale)
__global__ void flash_bwd_post_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv,
                                      int64_t T, int C, float scale) {
  const int64_t n = T * C / 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t t = (2 * i) / C;
    const int c = (int)((2 * i) % C);
    float2 v = reinterpret_cast<const float2*>(dq_acc)[i];
    *reinterpret_cast<uint32_t*>(dqkv + t * 3 * C + c) = pack_bf16x2(v.x * scale, v.y * scale);
  }
}

__global__ void __launch_bounds__(192, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                     const __grid_constant__ CUtensorMap tm_dout, const float* __restrict__ lse2,
                     const float* __restrict__ delta, float* __restrict__ dq_acc,
                     __nv_bfloat16* __restrict__ dqkv, const uint8_t* __restrict__ key_pad, int B,
                     int S, int H, int causal, float scale, uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int k0 = kt * kTile;
  const int C = H * kD;
  const int n_q_total = (S + kTile - 1) / kTile;
  const int qt_begin = causal ? kt : 0;
  const int n_it = n_q_total - qt_begin;
  const uint64_t limit = g_fa_wait_limit_ns;
  volatile uint32_t* abort_flag = &sm.abort;

  if (threadIdx.x == 0) {
    mbar_init(&sm.kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.qdo_full[i], 1);
      mbar_init(&sm.qdo_empty[i], 1);
    }
    mbar_init(&sm.sdp_full, 1);
    mbar_init(&sm.pds_ready, 4);
    mbar_init(&sm.dq_full, 1);
    mbar_init(&sm.dq_free, 4);
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  progress(1);
  if (warp == 1) {
    tmem_alloc<512>(&sm.tmem_base);
    tmem_relinquish();
  }
  progress(2);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 320,
                 t_dq = tmem + 384;

  if (warp == 0) {
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_qkv);
      tma_prefetch_desc(&tm_dout);
      mbar_arrive_expect_tx(&sm.kv_full, 2 * kTileBytes);
      tma_load_3d(sm.k, &tm_qkv, &sm.kv_full, C + h * kD, k0, b);
      tma_load_3d(sm.v, &tm_qkv, &sm.kv_full, 2 * C + h * kD, k0, b);
      for (int it = 0; it < n_it; ++it) {
        const int st = it & 1;
        const int qt = qt_begin + it;
        if (!mbar_wait_bounded(&sm.qdo_empty[st], ((it >> 1) & 1) ^ 1, abort_flag, err, limit))
          break;
        mbar_arrive_expect_tx(&sm.qdo_full[st], 2 * kTileBytes);
        tma_load_3d(sm.q[st], &tm_qkv, &sm.qdo_full[st], h * kD, qt * kTile, b);
        tma_load_3d(sm.dout[st], &tm_dout, &sm.qdo_full[st], h * kD, qt * kTile, b);
        progress(10 + it);
      }
      progress(19);
    }
    __syncwarp();  // reconverge the warp before the CTA-wide barrier below
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idesc_kq = make_idesc_bf16(128, 128, 0, 0);  // M=keys, N=queries
      constexpr uint32_t idesc_kd = make_idesc_bf16(128, kD, 0, 1);   // M=keys, N=D, B MN-major
      constexpr uint32_t idesc_qd = make_idesc_bf16(128, kD, 1, 1);   // M=queries, N=D, A,B MN-major
      const uint32_t k_addr = smem_u32(sm.k), v_addr = smem_u32(sm.v);
      const uint32_t p_addr = smem_u32(sm.p), ds_addr = smem_u32(sm.ds);
      bool ok = mbar_wait_bounded(&sm.kv_full, 0, abort_flag, err, limit);
      for (int it = 0; it < n_it && ok; ++it) {
        const int st = it & 1;
        ok = mbar_wait_bounded(&sm.qdo_full[st], (it >> 1) & 1, abort_flag, err, limit);
        if (!ok) break;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sm.q[st]), do_addr = smem_u32(sm.dout[st]);
        // S^T = K Q^T ; dP^T = V dO^T
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          umma_bf16(t_s, make_sdesc_sw128(k_addr + kk * 32, 16, 1024),
                    make_sdesc_sw128(q_addr + kk * 32, 16, 1024), idesc_kq, kk > 0);
          umma_bf16(t_dp, make_sdesc_sw128(v_addr + kk * 32, 16, 1024),
                    make_sdesc_sw128(do_addr + kk * 32, 16, 1024), idesc_kq, kk > 0);
        }
        umma_commit(&sm.sdp_full);
        progress(20 + 10 * it + 1);
        ok = mbar_wait_bounded(&sm.pds_ready, it & 1, abort_flag, err, limit);
        progress(20 + 10 * it + 2);
        if (!ok) break;
        tc_fence_after();
        // dV += P^T dO ; dK += dS^T Q   (K = 128 queries)
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint32_t aoff = (kk / 4) * kTileBytes + (kk % 4) * 32;
          umma_bf16(t_dv, make_sdesc_sw128(p_addr + aoff, 16, 1024),
                    make_sdesc_sw128(do_addr + kk * 2048, kTileBytes, 1024), idesc_kd,
                    (it > 0 || kk > 0));
          umma_bf16(t_dk, make_sdesc_sw128(ds_addr + aoff, 16, 1024),
                    make_sdesc_sw128(q_addr + kk * 2048, kTileBytes, 1024), idesc_kd,
                    (it > 0 || kk > 0));
        }
        if (it > 0) {
          ok = mbar_wait_bounded(&sm.dq_free, (it - 1) & 1, abort_flag, err, limit);
          if (!ok) break;
          tc_fence_after();
        }
        // dQ_i = dS K  (M = 128 queries, K = 128 keys): A = dS^T read MN-major
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_bf16(t_dq, make_sdesc_sw128(ds_addr + kk * 2048, kTileBytes, 1024),
                    make_sdesc_sw128(k_addr + kk * 2048, kTileBytes, 1024), idesc_qd, kk > 0);
        umma_commit(&sm.dq_full);
        umma_commit(&sm.qdo_empty[st]);
        progress(20 + 10 * it + 5);
      }
      progress(59);
      if (!ok) {
        umma_commit(&sm.drain);
        uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&sm.drain, 0) && global_timer_ns() - t0 < 100000000ull) {
        }
      }
    }
    __syncwarp();  // reconverge the warp before the CTA-wide barrier below
  } else {
    // --------------------------------------------------- softmax warps (thread = key row)
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const int kj = k0 + r;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float sl2 = scale * kLog2e;
    const bool key_ok = kj < S && !(key_pad && key_pad[(size_t)b * S + kj] != 0);
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int qt = qt_begin + it;
      const int q0 = qt * kTile;
      const float* lse_t = lse2 + ((size_t)b * H + h) * S + q0;
      const float* delta_t = delta + ((size_t)b * H + h) * S + q0;
      progress(60 + 10 * it);
      ok = mbar_wait_bounded(&sm.sdp_full, it & 1, abort_flag, err, limit);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      progress(60 + 10 * it + 1);
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < kTile; c += 32) {
        uint32_t rs[32], rdp[32];
        tmem_ld_32cols(t_s + lane_off + c, rs);
        tmem_ld_32cols(t_dp + lane_off + c, rdp);
        tmem_ld_wait();
        float pv[32], dsv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int qi = q0 + c + i;
          const bool valid = key_ok && qi < S && (!causal || kj <= qi);
          // per-query statistics: every thread reads the same words (L1 broadcast)
          const float l2 = qi < S ? __ldg(lse_t + c + i) : 0.f;
          const float dl = qi < S ? __ldg(delta_t + c + i) : 0.f;
          const float p = valid ? exp2f(__uint_as_float(rs[i]) * sl2 - l2) : 0.f;
          pv[i] = p;
          dsv[i] = p * (__uint_as_float(rdp[i]) - dl);
        }
        st_row32_sw128(sm.p, r, c, pv);
        st_row32_sw128(sm.ds, r, c, dsv);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.pds_ready);
      progress(60 + 10 * it + 2);
      // dQ tile: thread = query row (TMEM lane)
      ok = mbar_wait_bounded(&sm.dq_full, it & 1, abort_flag, err, limit);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      progress(60 + 10 * it + 3);
      tc_fence_after();
      {
        const int qi = q0 + r;
        float* dqrow = dq_acc + ((size_t)b * S + qi) * C + h * kD;
#pragma unroll
        for (int c = 0; c < kD; c += 32) {
          uint32_t raw[32];
          tmem_ld_32cols(t_dq + lane_off + c, raw);
          tmem_ld_wait();
          if (qi < S) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              red_add_v4(dqrow + c + i, __uint_as_float(raw[i]), __uint_as_float(raw[i + 1]),
                         __uint_as_float(raw[i + 2]), __uint_as_float(raw[i + 3]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.dq_free);
      progress(60 + 10 * it + 4);
    }
    progress(90);
    // dK, dV out (thread = key row). The last dq_full wait above implies all MMAs are done.
    if (ok && n_it > 0) {
      tc_fence_after();
      // tcgen05.ld is warp-synchronous: every lane loads, only in-range rows store
      __nv_bfloat16* krow = dqkv + ((size_t)b * S + kj) * 3 * C + C + h * kD;
      __nv_bfloat16* vrow = krow + C;
#pragma unroll
      for (int c = 0; c < kD; c += 32) {
        uint32_t rk[32], rv[32];
        tmem_ld_32cols(t_dk + lane_off + c, rk);
        tmem_ld_32cols(t_dv + lane_off + c, rv);
        tmem_ld_wait();
        if (kj < S) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 wk, wv;
            wk.x = pack_bf16x2(__uint_as_float(rk[8 * q + 0]) * scale, __uint_as_float(rk[8 * q + 1]) * scale);
            wk.y = pack_bf16x2(__uint_as_float(rk[8 * q + 2]) * scale, __uint_as_float(rk[8 * q + 3]) * scale);
            wk.z = pack_bf16x2(__uint_as_float(rk[8 * q + 4]) * scale, __uint_as_float(rk[8 * q + 5]) * scale);
            wk.w = pack_bf16x2(__uint_as_float(rk[8 * q + 6]) * scale, __uint_as_float(rk[8 * q + 7]) * scale);
            wv.x = pack_bf16x2(__uint_as_float(rv[8 * q + 0]), __uint_as_float(rv[8 * q + 1]));
            wv.y = pack_bf16x2(__uint_as_float(rv[8 * q + 2]), __uint_as_float(rv[8 * q + 3]));
            wv.z = pack_bf16x2(__uint_as_float(rv[8 * q + 4]), __uint_as_float(rv[8 * q + 5]));
            wv.w = pack_bf16x2(__uint_as_float(rv[8 * q + 6]), __uint_as_float(rv[8 * q + 7]));
            reinterpret_cast<uint4*>(krow + c)[q] = wk;
            reinterpret_cast<uint4*>(vrow + c)[q] = wv;
          }
        }
      }
    } else if (ok && kj < S) {
      // no query tile reaches this key tile: its gradients are zero
      __nv_bfloat16* krow = dqkv + ((size_t)b * S + kj) * 3 * C + C + h * kD;
      for (int c = 0; c < kD; ++c) {
        krow[c] = __float2bfloat16_rn(0.f);
        krow[C + c] = __float2bfloat16_rn(0.f);
      }
    }
  }
  progress(95);
  tc_fence_before();
  __syncthreads();
  progress(97);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
  progress(99);
}

}  // namespace

void set_flash_progress_words(uint32_t* dev_ptr) {
  cudaMemcpyToSymbol(g_fa_progress, &dev_ptr, sizeof(dev_ptr));
}

void set_flash_wait_limit_ns(uint64_t ns) {
  cudaMemcpyToSymbol(g_fa_wait_limit_ns, &ns, sizeof(ns));
}

cudaError_t launch_flash_fwd(const FlashArgs& a, cudaStream_t st) {
  if (a.D != kD || a.S <= 0 || a.B <= 0 || a.H <= 0) return cudaErrorInvalidValue;
  CUtensorMap tm;
  if (!make_map_3d(&tm, a.qkv, a.B, a.S, 3 * a.H * kD)) return cudaErrorInvalidValue;
  const int smem = (int)sizeof(FwdSmem) + 1024;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  dim3 grid((a.S + kTile - 1) / kTile, a.H, a.B);
  flash_fwd_kernel<<<grid, 192, smem, st>>>(tm, a.out, a.lse2, a.key_pad, a.B, a.S, a.H,
                                            a.causal ? 1 : 0, a.scale, a.err ? a.err : default_err_word());
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_flash_bwd(const FlashArgs& a, cudaStream_t st) {
  if (a.D != kD || a.S <= 0 || a.B <= 0 || a.H <= 0) return cudaErrorInvalidValue;
  const int C = a.H * kD;
  CUtensorMap tm_qkv, tm_do;
  if (!make_map_3d(&tm_qkv, a.qkv, a.B, a.S, 3 * C)) return cudaErrorInvalidValue;
  if (!make_map_3d(&tm_do, a.dout, a.B, a.S, C)) return cudaErrorInvalidValue;
  const int64_t rows = (int64_t)a.B * a.S * a.H;
  int pre_blocks = (int)std::min<int64_t>((rows + 7) / 8, (int64_t)num_sms() * 16);
  flash_bwd_pre_kernel<<<pre_blocks, 256, 0, st>>>(a.dout, a.out, a.delta, a.dq_acc, a.B, a.S, a.H);
  const int smem = (int)sizeof(BwdSmem) + 1024;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(flash_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  dim3 grid((a.S + kTile - 1) / kTile, a.H, a.B);
  flash_bwd_kernel<<<grid, 192, smem, st>>>(tm_qkv, tm_do, a.lse2, a.delta, a.dq_acc, a.dqkv,
                                            a.key_pad, a.B, a.S, a.H, a.causal ? 1 : 0, a.scale,
                                            a.err ? a.err : default_err_word());
  const int64_t T = (int64_t)a.B * a.S;
  int post_blocks = (int)std::min<int64_t>((T * C / 2 + 255) / 256, (int64_t)num_sms() * 16);
  flash_bwd_post_kernel<<<post_blocks, 256, 0, st>>>(a.dq_acc, a.dqkv, T, C, a.scale);
  note_launch(3);
  return cudaGetLastError();
}

}  // namespace flodl
