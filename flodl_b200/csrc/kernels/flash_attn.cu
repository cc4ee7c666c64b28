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

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace flodl {

namespace {

constexpr int kTile = 128;  // queries per fwd CTA, keys per bwd CTA, and the other tile dim
constexpr int kD = 64;
constexpr int kTileBytes = kTile * kD * 2;  // 16 KB: 128 rows x 128 B
constexpr float kLog2e = 1.4426950408889634f;

__device__ uint64_t g_fa_wait_limit_ns = 2000000000ull;
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
// Persistent: each CTA walks work items (128-query tile, head, batch) with a
// stride of gridDim.x, so Q/K/V loads and S MMAs of the next item overlap the
// softmax and output of the current one.
//
// Warps: 0 = TMA producer, 1 = MMA issuer, 2..9 = softmax. Softmax warp w owns
// TMEM lane quarter w & 3 (32 query rows) and column half (w - 2) / 4: 64 of
// the 128 keys of S, and 32 of the 64 columns of O. The two warps sharing a
// row set exchange partial row maxima through shared memory, synchronised by
// a per-pair mbarrier (bounded waits, never a named barrier, so an aborting
// warp cannot strand its partner).
//
// TMEM (512 columns): S double buffer at 0 / 128, O double buffer (by item
// parity) at 256 / 320. O accumulates P V across key tiles in TMEM. The
// running max is rescaled lazily: a row keeps its reference max until the new
// maximum exceeds it by more than 8 (log2 units), so P stays <= 2^8 and O is
// rescaled in TMEM only when the reference moves.
constexpr int kFwdSoftmaxWarps = 8;
constexpr int kFwdThreads = 64 + 32 * kFwdSoftmaxWarps;
constexpr float kRescaleThreshold = 8.0f;

struct FwdSmem {
  uint8_t q[2][kTileBytes];
  uint8_t k[2][kTileBytes];
  uint8_t v[2][kTileBytes];
  uint8_t p[2 * kTileBytes];        // P tile: 128 queries x 128 keys, two 64-key blocks
  float red_max[2][2][kTile];       // [tile parity][column half][row]
  float red_sum[2][kTile];          // [column half][row] final row sums
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[2], kv_empty[2];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full, pv_done;
  uint64_t o_full[2], o_free[2];
  uint64_t pair[4];                 // softmax warp pairs (per lane quarter)
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Work order: the tile index is the slowest-varying coordinate and, under a
// causal mask, the heaviest tiles (most key tiles) come first. CTA c takes
// items c, c + grid, ...; with the tile index fastest, an even grid would hand
// every CTA of one parity the same tile (all-heavy vs all-light CTAs), while
// heaviest-first striding gives each CTA a near-equal mix (longest-processing-
// time-first list scheduling).
__device__ __forceinline__ void fwd_decode(int item, int n_qt, int H, int n_bh, bool causal,
                                           int& qt, int& h, int& b) {
  const int t = item / n_bh;
  const int bh = item - t * n_bh;
  qt = causal ? n_qt - 1 - t : t;
  h = bh % H;
  b = bh / H;
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, __nv_bfloat16* __restrict__ out,
                     float* __restrict__ lse2, const uint8_t* __restrict__ key_pad, int B, int S,
                     int H, int causal, float scale, uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  FwdSmem& sm = *reinterpret_cast<FwdSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int C = H * kD;
  const int n_qt = (S + kTile - 1) / kTile;
  const int n_items = n_qt * H * B;
  const uint64_t limit = g_fa_wait_limit_ns;
  volatile uint32_t* abort_flag = &sm.abort;
  auto kv_tiles = [&](int qt) { return causal ? min(qt + 1, n_qt) : n_qt; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.q_full[i], 1);
      mbar_init(&sm.q_empty[i], 1);
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], kFwdSoftmaxWarps);
      mbar_init(&sm.o_full[i], 1);
      mbar_init(&sm.o_free[i], kFwdSoftmaxWarps);
    }
    mbar_init(&sm.p_full, kFwdSoftmaxWarps);
    mbar_init(&sm.pv_done, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&sm.pair[i], 64);
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<512>(&sm.tmem_base);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  pdl_wait();  // global memory only after the previous kernel of the stream
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_qkv);
      uint32_t kv_it = 0;
      bool ok = true;
      int n = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
        int qt, h, b;
        fwd_decode(item, n_qt, H, H * B, causal != 0, qt, h, b);
        const int qb = n & 1;
        if (!(ok = mbar_wait_bounded(&sm.q_empty[qb], ((n >> 1) & 1) ^ 1, abort_flag, err, limit)))
          break;
        mbar_arrive_expect_tx(&sm.q_full[qb], kTileBytes);
        tma_load_3d(sm.q[qb], &tm_qkv, &sm.q_full[qb], h * kD, qt * kTile, b);
        const int nkv = kv_tiles(qt);
        for (int j = 0; j < nkv; ++j, ++kv_it) {
          const int st = kv_it & 1;
          if (!(ok = mbar_wait_bounded(&sm.kv_empty[st], ((kv_it >> 1) & 1) ^ 1, abort_flag, err,
                                       limit)))
            break;
          mbar_arrive_expect_tx(&sm.kv_full[st], 2 * kTileBytes);
          tma_load_3d(sm.k[st], &tm_qkv, &sm.kv_full[st], C + h * kD, j * kTile, b);
          tma_load_3d(sm.v[st], &tm_qkv, &sm.kv_full[st], 2 * C + h * kD, j * kTile, b);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(128, kD, 0, 1);
      const uint32_t p_addr = smem_u32(sm.p);
      uint32_t kv_it = 0, s_it = 0, p_it = 0;
      bool ok = true, issued = false;
      int n = 0;
      auto issue_pv = [&](uint32_t kv_stage, uint32_t t_o, bool acc) -> bool {
        if (!mbar_wait_bounded(&sm.p_full, p_it & 1, abort_flag, err, limit)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm.v[kv_stage]);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint64_t a =
              make_sdesc_sw128(p_addr + (kk / 4) * kTileBytes + (kk % 4) * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(v_addr + kk * 2048, kTileBytes, 1024);
          umma_bf16(t_o, a, bd, idesc_o, (acc || kk > 0) ? 1u : 0u);
        }
        umma_commit(&sm.pv_done);
        umma_commit(&sm.kv_empty[kv_stage]);
        ++p_it;
        return true;
      };
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
        int qt, h, b;
        fwd_decode(item, n_qt, H, H * B, causal != 0, qt, h, b);
        const int qb = n & 1;
        const uint32_t t_o = tmem + 256 + (uint32_t)qb * kD;
        if (!(ok = mbar_wait_bounded(&sm.q_full[qb], (n >> 1) & 1, abort_flag, err, limit))) break;
        if (!(ok = mbar_wait_bounded(&sm.o_free[qb], ((n >> 1) & 1) ^ 1, abort_flag, err, limit)))
          break;
        const uint32_t q_addr = smem_u32(sm.q[qb]);
        const int nkv = kv_tiles(qt);
        uint32_t prev_stage = 0;
        for (int j = 0; j < nkv && ok; ++j, ++kv_it, ++s_it) {
          const uint32_t st = kv_it & 1, sb = s_it & 1;
          if (!(ok = mbar_wait_bounded(&sm.kv_full[st], (kv_it >> 1) & 1, abort_flag, err, limit)))
            break;
          if (!(ok = mbar_wait_bounded(&sm.s_free[sb], ((s_it >> 1) & 1) ^ 1, abort_flag, err,
                                       limit)))
            break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sm.k[st]);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            umma_bf16(tmem + sb * 128, make_sdesc_sw128(q_addr + kk * 32, 16, 1024),
                      make_sdesc_sw128(k_addr + kk * 32, 16, 1024), idesc_s, kk > 0);
          issued = true;
          umma_commit(&sm.s_full[sb]);
          if (j == nkv - 1) umma_commit(&sm.q_empty[qb]);  // Q no longer read
          // P V of the previous key tile overlaps this S
          if (j > 0 && !(ok = issue_pv(prev_stage, t_o, j > 1))) break;
          prev_stage = st;
        }
        if (!ok) break;
        if (!(ok = issue_pv(prev_stage, t_o, nkv > 1))) break;
        umma_commit(&sm.o_full[qb]);
      }
      if (!ok && issued) {
        umma_commit(&sm.drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&sm.drain, 0) && global_timer_ns() - t0 < 100000000ull) {
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int q4 = warp & 3;
    const int hh = (warp - 2) >> 2;  // column half
    const int r = q4 * 32 + lane;    // query row within the tile
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float sl2 = scale * kLog2e;
    uint64_t* pair = &sm.pair[q4];
    uint32_t s_it = 0, p_it = 0, pair_it = 0;
    bool ok = true;
    int n = 0;
    // pair exchange: every lane arrives, then waits for the partner warp
    auto pair_sync = [&]() -> bool {
      mbar_arrive(pair);
      const bool w = mbar_wait_bounded(pair, pair_it & 1, abort_flag, err, limit);
      ++pair_it;
      return __all_sync(0xffffffffu, w);
    };
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
      int qt, h, b;
      fwd_decode(item, n_qt, H, H * B, causal != 0, qt, h, b);
      const int qb = n & 1;
      const uint32_t t_o = tmem + 256 + (uint32_t)qb * kD;
      const int q0 = qt * kTile;
      const int qi = q0 + r;
      const int nkv = kv_tiles(qt);
      float m_ref = -INFINITY;  // reference max (scaled, log2 units)
      float l_half = 0.f;       // this warp's partial row sum
      for (int j = 0; j < nkv; ++j, ++s_it, ++p_it) {
        const uint32_t sb = s_it & 1;
        ok = mbar_wait_bounded(&sm.s_full[sb], (s_it >> 1) & 1, abort_flag, err, limit);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        float s[64];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t raw[32];
          tmem_ld_32cols(tmem + sb * 128 + lane_off + (uint32_t)(hh * 64 + c * 32), raw);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; i += 2)
            f2_unpack(f2_mul(f2_pack(__uint_as_float(raw[i]), __uint_as_float(raw[i + 1])),
                             f2_splat(sl2)),
                      s[c * 32 + i], s[c * 32 + i + 1]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_free[sb]);
        // masks: key range, causal diagonal, key padding
        const int k0 = j * kTile + hh * 64;
        const bool diag = causal && (k0 + 63 > q0);
        const bool tail = (k0 + 64 > S);
        if (diag || tail || key_pad) {
          uint32_t padw[16];
          if (key_pad) {
            const uint8_t* kp = key_pad + (size_t)b * S + k0;
#pragma unroll
            for (int w4 = 0; w4 < 16; ++w4) {
              uint32_t word = 0;
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const int kj = k0 + w4 * 4 + t;
                const uint32_t mbyte = (kj < S) ? (uint32_t)__ldg(kp + w4 * 4 + t) : 1u;
                word |= (mbyte ? 1u : 0u) << (8 * t);
              }
              padw[w4] = word;
            }
          }
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const int kj = k0 + c;
            bool valid = kj < S && (!causal || kj <= qi);
            if (key_pad) valid = valid && !((padw[c >> 2] >> (8 * (c & 3))) & 0xffu);
            if (!valid) s[c] = -INFINITY;
          }
        }
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], s[c]);
        const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        sm.red_max[j & 1][hh][r] = mx;
        if (!pair_sync()) { ok = false; break; }
        const float m_tile = fmaxf(mx, sm.red_max[j & 1][hh ^ 1][r]);
        // lazy rescale: move the reference only when the max grew by > threshold
        const bool move = m_tile > m_ref + kRescaleThreshold;
        const float m_new = move ? m_tile : m_ref;
        const float corr = (move && m_ref != -INFINITY) ? ex2_approx(m_ref - m_new) : 1.f;
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        m_ref = m_new;
        uint64_t l2a = f2_splat(0.f), l2b = f2_splat(0.f);
        const uint64_t neg_m = f2_splat(-m_use);
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          float a0, a1;
          f2_unpack(f2_add(f2_pack(s[c], s[c + 1]), neg_m), a0, a1);
          s[c] = ex2_approx(a0);
          s[c + 1] = ex2_approx(a1);
          if (c & 2)
            l2b = f2_add(l2b, f2_pack(s[c], s[c + 1]));
          else
            l2a = f2_add(l2a, f2_pack(s[c], s[c + 1]));
        }
        float la0, la1, lb0, lb1;
        f2_unpack(l2a, la0, la1);
        f2_unpack(l2b, lb0, lb1);
        l_half = l_half * corr + ((la0 + la1) + (lb0 + lb1));
        // P is single-buffered: the previous P V must have finished reading it
        if (p_it > 0) {
          ok = mbar_wait_bounded(&sm.pv_done, (p_it - 1) & 1, abort_flag, err, limit);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          tc_fence_after();
        }
        // rescale this warp's 32 columns of O when any of its rows moved
        if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
          const uint32_t taddr = t_o + lane_off + (uint32_t)(hh * 32);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t o[16];
            tmem_ld_16cols(taddr + c * 16, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
            tmem_st_16cols(taddr + c * 16, o);
          }
          tmem_st_wait();
        }
        // P (bf16) -> this warp's 64-key block of the SW128 K-major P tile
        uint8_t* blk = sm.p + hh * kTileBytes;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint4 w;
          w.x = pack_bf16x2(s[8 * q + 0], s[8 * q + 1]);
          w.y = pack_bf16x2(s[8 * q + 2], s[8 * q + 3]);
          w.z = pack_bf16x2(s[8 * q + 4], s[8 * q + 5]);
          w.w = pack_bf16x2(s[8 * q + 6], s[8 * q + 7]);
          st_sw128_chunk(blk, r, q, w);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full);
      }
      if (!ok) break;
      // ---- output of this item: O / l for this warp's 32 columns, and lse
      sm.red_sum[hh][r] = l_half;
      if (!pair_sync()) { ok = false; break; }
      const float l = l_half + sm.red_sum[hh ^ 1][r];
      ok = mbar_wait_bounded(&sm.o_full[qb], (n >> 1) & 1, abort_flag, err, limit);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      uint32_t o[32];
      tmem_ld_32cols(t_o + lane_off + (uint32_t)(hh * 32), o);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.o_free[qb]);
      if (qi < S) {
        const float inv_l = l > 0.f ? 1.f / l : 0.f;
        uint4* orow = reinterpret_cast<uint4*>(out + ((size_t)b * S + qi) * C + h * kD + hh * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l);
          w.y = pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l);
          w.z = pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l);
          w.w = pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l);
          orow[q] = w;
        }
        if (hh == 0)
          lse2[((size_t)b * H + h) * S + qi] = (l > 0.f) ? (m_ref + log2f(l)) : -INFINITY;
      }
      // the red_sum slot is rewritten next item only after the pair passes
      // at least one more pair_sync (the first max exchange), so no extra sync
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

// ============================================================== forward, two CTAs per SM
// The same computation with one query row per thread and P kept in tensor
// memory. Two CTAs share each SM (97 KB of shared memory, 256 TMEM columns
// and 192 threads each): inside a CTA the chain S -> softmax -> P V is serial
// per key tile, and the other CTA's MMAs, loads and softmax fill its gaps.
//
// Warps: 0 = TMA producer, 1 = MMA issuer, 2..5 = softmax. Softmax warp w owns
// TMEM lane quarter w & 3; a thread owns one query row and all 128 keys of a
// tile, so no exchange between warps is needed. The row maximum takes a first
// pass over S (32 columns at a time), the exponentials a second pass.
//
// TMEM (256 columns): S at 0 (128 columns). The softmax writes P (bf16 pairs,
// 64 columns) over S in place: P columns [16c, 16c + 16) replace S columns
// that pass c has already read. The P V MMA takes P as its A operand straight
// from TMEM. O double buffer (by item parity) at 128 / 192, rescaled lazily
// in TMEM like the 8-warp kernel. The MMAs of one thread execute in issue
// order, so S of the next key tile, issued after P V, cannot overwrite P
// before P V has read it; and the commit that signals S(j) also covers P V of
// tile j-1, so a rescale of O never races an MMA.
constexpr int kF2Warps = 4;
constexpr int kF2Threads = 64 + 32 * kF2Warps;

struct Fwd2Smem {
  uint8_t q[2][kTileBytes];
  uint8_t k[2][kTileBytes];
  uint8_t v[2][kTileBytes];
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[2], kv_empty[2];
  uint64_t s_full, p_full;
  uint64_t o_full[2], o_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};

// Key-padding mask of 32 columns: -inf where the key is padded (BERT-style
// batches; the causal/range part is handled by the per-row limit).
__device__ __forceinline__ void f2_pad_mask32(float (&v)[32], int kc0, int S,
                                              const uint8_t* kp_row) {
#pragma unroll
  for (int w4 = 0; w4 < 8; ++w4) {
    const int k = kc0 + 4 * w4;
    uint32_t word;
    if (k + 3 < S && ((reinterpret_cast<uintptr_t>(kp_row + k) & 3) == 0)) {
      word = __ldg(reinterpret_cast<const uint32_t*>(kp_row + k));
    } else {
      word = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t)
        word |= (uint32_t)((k + t < S) ? __ldg(kp_row + k + t) : 0) << (8 * t);
    }
#pragma unroll
    for (int t = 0; t < 4; ++t)
      if ((word >> (8 * t)) & 0xffu) v[4 * w4 + t] = -INFINITY;
  }
}

// Key padding of one 128-key tile as a suffix, found once per tile by a warp:
// lane l reads keys k0 + 4l .. k0 + 4l + 3 (keys at or past S count as
// padded). Returns the first padded key's offset in the tile (128: none) when
// every key from it on is padded - right-padded batches, which then need no
// per-key mask, only a shorter row limit - and -1 when the tile mixes padded
// and unpadded keys after the first padded one.
__device__ __forceinline__ int f2_pad_suffix(const uint8_t* kp_row, int k0, int S, int lane) {
  const int k = k0 + 4 * lane;
  uint32_t word = 0;
  if (k + 3 < S && ((reinterpret_cast<uintptr_t>(kp_row + k) & 3) == 0)) {
    word = __ldg(reinterpret_cast<const uint32_t*>(kp_row + k));
  } else {
#pragma unroll
    for (int t = 0; t < 4; ++t)
      word |= (uint32_t)((k + t < S) ? __ldg(kp_row + k + t) : 1) << (8 * t);
  }
  uint32_t pad = 0;  // bit t: key k + t padded
#pragma unroll
  for (int t = 0; t < 4; ++t) pad |= (((word >> (8 * t)) & 0xffu) != 0 ? 1u : 0u) << t;
  const uint32_t any = __ballot_sync(0xffffffffu, pad != 0);
  if (any == 0) return kTile;
  const int L = __ffs(any) - 1;  // first lane holding a padded key
  const uint32_t full = __ballot_sync(0xffffffffu, pad == 0xfu);
  const int first = __ffs(__shfl_sync(0xffffffffu, pad, L)) - 1;
  const uint32_t lpad = __shfl_sync(0xffffffffu, pad, L);
  // lane L padded from its first padded key on, every later lane fully padded
  const bool tail_ok = (lpad >> first) == (0xfu >> first);
  const uint32_t later = L == 31 ? 0u : (0xffffffffu << (L + 1));
  return (tail_ok && (full & later) == later) ? 4 * L + first : -1;
}

__global__ void __launch_bounds__(kF2Threads, 2)
    flash_fwd2_kernel(const __grid_constant__ CUtensorMap tm_qkv, __nv_bfloat16* __restrict__ out,
                      float* __restrict__ lse2, const uint8_t* __restrict__ key_pad, int B, int S,
                      int H, int causal, float scale, uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Fwd2Smem& sm = *reinterpret_cast<Fwd2Smem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int C = H * kD;
  const int n_qt = (S + kTile - 1) / kTile;
  const int n_items = n_qt * H * B;
  const uint64_t limit = g_fa_wait_limit_ns;
  volatile uint32_t* abort_flag = &sm.abort;
  auto kv_tiles = [&](int qt) { return causal ? min(qt + 1, n_qt) : n_qt; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.q_full[i], 1);
      mbar_init(&sm.q_empty[i], 1);
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
      mbar_init(&sm.o_full[i], 1);
      mbar_init(&sm.o_free[i], kF2Warps);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.p_full, kF2Warps);
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
  pdl_wait();  // global memory only after the previous kernel of the stream
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_qkv);
      uint32_t kv_it = 0;
      bool ok = true;
      int n = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
        int qt, h, b;
        fwd_decode(item, n_qt, H, H * B, causal != 0, qt, h, b);
        const int qb = n & 1;
        if (!(ok = mbar_wait_bounded(&sm.q_empty[qb], ((n >> 1) & 1) ^ 1, abort_flag, err, limit)))
          break;
        mbar_arrive_expect_tx(&sm.q_full[qb], kTileBytes);
        tma_load_3d(sm.q[qb], &tm_qkv, &sm.q_full[qb], h * kD, qt * kTile, b);
        const int nkv = kv_tiles(qt);
        for (int j = 0; j < nkv; ++j, ++kv_it) {
          const int st = kv_it & 1;
          if (!(ok = mbar_wait_bounded(&sm.kv_empty[st], ((kv_it >> 1) & 1) ^ 1, abort_flag, err,
                                       limit)))
            break;
          mbar_arrive_expect_tx(&sm.kv_full[st], 2 * kTileBytes);
          tma_load_3d(sm.k[st], &tm_qkv, &sm.kv_full[st], C + h * kD, j * kTile, b);
          tma_load_3d(sm.v[st], &tm_qkv, &sm.kv_full[st], 2 * C + h * kD, j * kTile, b);
        }
      }
    }
    __syncwarp();  // reconverge before the CTA-wide barrier at the end
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(128, kD, 0, 1);
      uint32_t kv_it = 0, t_it = 0;
      bool ok = true, issued = false;
      int n = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
        int qt, h, b;
        fwd_decode(item, n_qt, H, H * B, causal != 0, qt, h, b);
        const int qb = n & 1;
        const uint32_t t_o = tmem + 128 + (uint32_t)qb * kD;
        if (!(ok = mbar_wait_bounded(&sm.q_full[qb], (n >> 1) & 1, abort_flag, err, limit))) break;
        const uint32_t q_addr = smem_u32(sm.q[qb]);
        const int nkv = kv_tiles(qt);
        for (int j = 0; j < nkv; ++j, ++kv_it, ++t_it) {
          const uint32_t st = kv_it & 1;
          if (!(ok = mbar_wait_bounded(&sm.kv_full[st], (kv_it >> 1) & 1, abort_flag, err, limit)))
            break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sm.k[st]);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            umma_bf16(tmem, make_sdesc_sw128(q_addr + kk * 32, 16, 1024),
                      make_sdesc_sw128(k_addr + kk * 32, 16, 1024), idesc_s, kk > 0);
          issued = true;
          umma_commit(&sm.s_full);
          if (j == nkv - 1) umma_commit(&sm.q_empty[qb]);  // Q no longer read
          // the O buffer of this parity was read out (item n - 2)
          if (j == 0 && !(ok = mbar_wait_bounded(&sm.o_free[qb], ((n >> 1) & 1) ^ 1, abort_flag,
                                                 err, limit)))
            break;
          // P (written over S by the softmax) times V
          if (!(ok = mbar_wait_bounded(&sm.p_full, t_it & 1, abort_flag, err, limit))) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sm.v[st]);
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk)
            umma_bf16_tmem_a(t_o, tmem + (uint32_t)(kk * 8),
                             make_sdesc_sw128(v_addr + kk * 2048, kTileBytes, 1024), idesc_o,
                             (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&sm.kv_empty[st]);
        }
        if (!ok) break;
        umma_commit(&sm.o_full[qb]);
      }
      if (!ok && issued) {
        umma_commit(&sm.drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&sm.drain, 0) && global_timer_ns() - t0 < 100000000ull) {
        }
      }
    }
    __syncwarp();  // reconverge before the CTA-wide barrier at the end
  } else {
    // ------------------------------------------------------------ softmax
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t t_s = tmem + lane_off;
    const float sl2 = scale * kLog2e;
    uint32_t t_it = 0;
    bool ok = true;
    int n = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
      int qt, h, b;
      fwd_decode(item, n_qt, H, H * B, causal != 0, qt, h, b);
      const int qb = n & 1;
      const uint32_t t_o = tmem + 128 + (uint32_t)qb * kD + lane_off;
      const int q0 = qt * kTile;
      const int qi = q0 + r;
      const int nkv = kv_tiles(qt);
      const uint8_t* kp_row = key_pad ? key_pad + (size_t)b * S : nullptr;
      float m_ref = -INFINITY;  // reference max (scaled, log2 units)
      float l = 0.f;            // row sum relative to m_ref
      for (int j = 0; j < nkv; ++j, ++t_it) {
        ok = mbar_wait_bounded(&sm.s_full, t_it & 1, abort_flag, err, limit);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        const int k0 = j * kTile;
        // right padding of this tile as a shorter row limit; a tile whose
        // padding is not a suffix keeps the per-key mask
        const int pad_from = kp_row ? f2_pad_suffix(kp_row, k0, S, lane) : kTile;
        const uint8_t* kp_mask = pad_from < 0 ? kp_row : nullptr;
        // valid keys of this row in this tile: [k0, k0 + lim) (range, causal, padding)
        const int lim = max(0, min(min((causal ? min(qi + 1, S) : S) - k0, kTile),
                                   pad_from < 0 ? kTile : pad_from));
        const bool ranged = lim < kTile;  // warp-uniform only on tiles without masking
        // pass 1: row maximum of the raw scores (scale > 0 commutes with max),
        // 64 columns per tensor-memory round trip
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t raw[2][32];
          tmem_ld_32cols(t_s + (uint32_t)(c2 * 64), raw[0]);
          tmem_ld_32cols(t_s + (uint32_t)(c2 * 64 + 32), raw[1]);
          tmem_ld_wait();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = c2 * 2 + h;
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[h][i]);
            if (ranged) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = (c * 32 + i < lim) ? v[i] : -INFINITY;
            }
            if (kp_mask) f2_pad_mask32(v, k0 + c * 32, S, kp_mask);
#pragma unroll
            for (int i = 0; i < 32; ++i) m4[i & 3] = fmaxf(m4[i & 3], v[i]);
          }
        }
        const float mraw = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        const float mx = mraw == -INFINITY ? -INFINITY : mraw * sl2;
        // lazy rescale: move the reference only when the max grew by > threshold
        const bool move = mx > m_ref + kRescaleThreshold;
        const float m_new = move ? mx : m_ref;
        const float corr = (move && m_ref != -INFINITY) ? ex2_approx(m_ref - m_new) : 1.f;
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        m_ref = m_new;
        // pass 2: P = 2^(s * scale - m) as bf16 over S (masked keys 0), row sum
        const uint64_t neg_m = f2_splat(-m_use);
        const uint64_t sl2x2 = f2_splat(sl2);
        uint64_t la = f2_splat(0.f), lb = f2_splat(0.f);
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          // 64 columns per round trip; P of these columns lands in columns
          // [32 c2, 32 c2 + 32), which hold scores already in registers
          uint32_t raw2[2][32];
          tmem_ld_32cols(t_s + (uint32_t)(c2 * 64), raw2[0]);
          tmem_ld_32cols(t_s + (uint32_t)(c2 * 64 + 32), raw2[1]);
          tmem_ld_wait();
#pragma unroll
          for (int hc = 0; hc < 2; ++hc) {
            const int c = c2 * 2 + hc;
            const uint32_t (&raw)[32] = raw2[hc];
            float p[32];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float a0, a1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(raw[i]), __uint_as_float(raw[i + 1])),
                               sl2x2, neg_m),
                        a0, a1);
              p[i] = ex2_approx(a0);
              p[i + 1] = ex2_approx(a1);
            }
            if (ranged) {
#pragma unroll
              for (int i = 0; i < 32; ++i) p[i] = (c * 32 + i < lim) ? p[i] : 0.f;
            }
            if (kp_mask) {
              float v[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = 0.f;
              f2_pad_mask32(v, k0 + c * 32, S, kp_mask);
#pragma unroll
              for (int i = 0; i < 32; ++i) p[i] = v[i] == -INFINITY ? 0.f : p[i];
            }
            uint32_t pw[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              if (i & 2)
                lb = f2_add(lb, f2_pack(p[i], p[i + 1]));
              else
                la = f2_add(la, f2_pack(p[i], p[i + 1]));
              pw[i / 2] = pack_bf16x2(p[i], p[i + 1]);
            }
            tmem_st_16cols(t_s + (uint32_t)(c * 16), pw);
          }
        }
        float la0, la1, lb0, lb1;
        f2_unpack(la, la0, la1);
        f2_unpack(lb, lb0, lb1);
        l = l * corr + ((la0 + la1) + (lb0 + lb1));
        // rescale O when a row's reference moved (P V of tile j - 1 is complete:
        // the commit behind s_full follows it)
        if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
          for (int c = 0; c < kD / 16; ++c) {
            uint32_t o[16];
            tmem_ld_16cols(t_o + (uint32_t)(c * 16), o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
            tmem_st_16cols(t_o + (uint32_t)(c * 16), o);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full);
      }
      if (!ok) break;
      // ---- output of this item: O / l and lse
      ok = mbar_wait_bounded(&sm.o_full[qb], (n >> 1) & 1, abort_flag, err, limit);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      uint32_t o[2][32];
      tmem_ld_32cols(t_o, o[0]);
      tmem_ld_32cols(t_o + 32, o[1]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.o_free[qb]);
      if (qi < S) {
        const float inv_l = l > 0.f ? 1.f / l : 0.f;
        uint4* orow = reinterpret_cast<uint4*>(out + ((size_t)b * S + qi) * C + h * kD);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t* oo = &o[q >> 2][(q & 3) * 8];
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(oo[0]) * inv_l, __uint_as_float(oo[1]) * inv_l);
          w.y = pack_bf16x2(__uint_as_float(oo[2]) * inv_l, __uint_as_float(oo[3]) * inv_l);
          w.z = pack_bf16x2(__uint_as_float(oo[4]) * inv_l, __uint_as_float(oo[5]) * inv_l);
          w.w = pack_bf16x2(__uint_as_float(oo[6]) * inv_l, __uint_as_float(oo[7]) * inv_l);
          orow[q] = w;
        }
        lse2[((size_t)b * H + h) * S + qi] = (l > 0.f) ? (m_ref + log2f(l)) : -INFINITY;
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
// Persistent over work items (128-key tile, head, batch). Per item the CTA
// walks the query tiles that see these keys (all, or those at/after the key
// tile when causal):
//   S^T = K Q_i^T, dP^T = V dO_i^T                        (TMEM, 128 x 128 each)
//   P^T = exp2(S^T * scale * log2e - lse2_i), dS^T = P^T (dP^T - delta_i)
//   dV += P^T dO_i, dK += dS^T Q_i                         (TMEM accumulators)
//   dQ_i = dS K -> f32 red.add into the dQ accumulator      (TMEM, read out one tile late)
// Warps: 0 = TMA producer, 1 = MMA issuer, 2..9 = compute. Compute warp w owns
// key rows 32 (w & 3) .. +31 (its TMEM lane quarter) and query half (w - 2) / 4
// of each tile (64 columns of S^T / dP^T, 32 columns of dQ / dK / dV). The
// halves need no exchange: the softmax statistics come precomputed (lse2,
// delta). TMEM: S^T 0, dP^T 128, dV 256, dK 320, dQ 384 (512 allocated).
constexpr int kBwdWarps = 8;
constexpr int kBwdThreads = 64 + 32 * kBwdWarps;

struct BwdSmem {
  uint8_t k[2][kTileBytes];  // K/V of two work items: the next item's tile
  uint8_t v[2][kTileBytes];  // loads while this item runs
  uint8_t q[2][kTileBytes];
  uint8_t dout[2][kTileBytes];
  uint8_t p[2 * kTileBytes];   // P^T: 128 keys x 128 queries (two 64-query SW128 blocks)
  uint8_t ds[2 * kTileBytes];  // dS^T, same layout
  float stat[kBwdWarps][2][64];  // per compute warp: lse2 and delta of its 64 queries
  uint64_t kv_full[2], kv_empty[2];
  uint64_t qdo_full[2], qdo_empty[2];
  uint64_t s_full, s_free, p_ready, pds_free, dq_full, dq_free, dkv_full, dkv_free;
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};

// delta[b,h,s] = sum_d dO * O ; also zeroes the f32 dQ accumulator rows
// (when there is one: the per-(batch, head) kernel keeps dQ in TMEM).
// A warp handles four (token, head) rows per step: eight lanes per row, each
// with 16-byte loads of dO and O (8 values) and a 3-step shuffle reduction.
__global__ void flash_bwd_pre_kernel(const __nv_bfloat16* __restrict__ dout,
                                     const __nv_bfloat16* __restrict__ out, float* __restrict__ delta,
                                     float* __restrict__ dq_acc, int B, int S, int H) {
  pdl_wait();
  pdl_trigger();
  // row rw = token * H + head is the contiguous 64-element slice at rw * kD
  // (B * S * H < 2^31, checked by the launcher); 8 lanes per row
  const int rows = B * S * H;
  const int warp_g = (int)((blockIdx.x * blockDim.x + threadIdx.x) / 32);
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 3, part = lane & 7;
  const int nw = (int)(gridDim.x * blockDim.x / 32);
#pragma unroll 2
  for (int base = warp_g * 4; base < rows; base += nw * 4) {
    const int rw = base + sub;
    float s = 0.f;
    if (rw < rows) {
      const int64_t off = (int64_t)rw * kD + part * 8;
      const uint4 x = *reinterpret_cast<const uint4*>(dout + off);
      const uint4 y = *reinterpret_cast<const uint4*>(out + off);
      const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 a = unpack_bf16x2(xs[k]), c = unpack_bf16x2(ys[k]);
        s = fmaf(a.x, c.x, fmaf(a.y, c.y, s));
      }
      if (dq_acc != nullptr) {
        float4* dq = reinterpret_cast<float4*>(dq_acc + off);
        dq[0] = make_float4(0.f, 0.f, 0.f, 0.f);
        dq[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (rw < rows && part == 0) {
      const int tok = rw / H, h = rw - tok * H;
      const int bb = tok / S, si = tok - bb * S;
      delta[((int64_t)bb * H + h) * S + si] = s;
    }
  }
}

// dqkv[:, q cols] = bf16(dq_acc * scale). With dbias, also the Q part of the
// packed projection's bias gradient: dbias[c] += sum over rows of the bf16 dQ
// for the C query columns, one atomic per column and row slice (the main
// kernel adds the K and V parts while it reads dK/dV out of TMEM). Thread = 8
// consecutive columns of a row; a block is `lanes` row lanes of `gw` threads
// each (gw = the C/8 column groups rounded up to a warp).
constexpr int kPostMaxThreads = 1024;
__global__ void __launch_bounds__(kPostMaxThreads) flash_bwd_post_kernel(
    const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv, int T, int C, float scale,
    float* __restrict__ dbias, int rows_per_block, int gw) {
  pdl_wait();
  pdl_trigger();
  const int groups = C / 8;  // dQ columns (the K/V bias sums come from the main kernel)
  const int lanes = blockDim.x / gw;
  const int g = blockIdx.y * gw + (int)(threadIdx.x % gw);
  const int rl = (int)(threadIdx.x / gw);  // row lane
  const int c0 = g * 8;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(T, r0 + rows_per_block);
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  if (g < groups) {
#pragma unroll 4
    for (int r = r0 + rl; r < r1; r += lanes) {
      uint4* dst = reinterpret_cast<uint4*>(dqkv + (size_t)r * 3 * C + c0);
      uint4 w;
      const float4* src = reinterpret_cast<const float4*>(dq_acc + (size_t)r * C + c0);
      const float4 a = src[0], b = src[1];
      w.x = pack_bf16x2(a.x * scale, a.y * scale);
      w.y = pack_bf16x2(a.z * scale, a.w * scale);
      w.z = pack_bf16x2(b.x * scale, b.y * scale);
      w.w = pack_bf16x2(b.z * scale, b.w * scale);
      *dst = w;
      if (dbias) {
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 f = unpack_bf16x2(ws[h]);
          acc[2 * h] += f.x;
          acc[2 * h + 1] += f.y;
        }
      }
    }
  }
  if (dbias == nullptr) return;  // uniform across the block
  __shared__ float red[kPostMaxThreads][9];
#pragma unroll
  for (int e = 0; e < 8; ++e) red[threadIdx.x][e] = acc[e];
  __syncthreads();
  if (rl == 0 && g < groups) {
    for (int l = 1; l < lanes; ++l)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += red[threadIdx.x + gw * l][e];
#pragma unroll
    for (int e = 0; e < 8; ++e) atomicAdd(dbias + c0 + e, acc[e]);
  }
}

// Same order as the forward: tile slowest; under a causal mask key tile 0
// sees every query tile, so ascending key tiles are heaviest-first.
__device__ __forceinline__ void bwd_decode(int item, int n_bh, int H, int& kt, int& h, int& b) {
  kt = item / n_bh;
  const int bh = item - kt * n_bh;
  h = bh % H;
  b = bh / H;
}

__global__ void __launch_bounds__(kBwdThreads, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                     const __grid_constant__ CUtensorMap tm_dout, const float* __restrict__ lse2,
                     const float* __restrict__ delta, float* __restrict__ dq_acc,
                     __nv_bfloat16* __restrict__ dqkv, const uint8_t* __restrict__ key_pad, int B,
                     int S, int H, int causal, float scale, float* __restrict__ dbias,
                     uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int C = H * kD;
  const int n_t = (S + kTile - 1) / kTile;  // tiles along the sequence
  const int n_items = n_t * H * B;
  const uint64_t limit = g_fa_wait_limit_ns;
  volatile uint32_t* abort_flag = &sm.abort;
  auto first_q = [&](int kt) { return causal ? kt : 0; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.qdo_full[i], 1);
      mbar_init(&sm.qdo_empty[i], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, kBwdWarps);
    mbar_init(&sm.p_ready, kBwdWarps);
    mbar_init(&sm.pds_free, 1);
    mbar_init(&sm.dq_full, 1);
    mbar_init(&sm.dq_free, kBwdWarps);
    mbar_init(&sm.dkv_full, 1);
    mbar_init(&sm.dkv_free, kBwdWarps);
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<512>(&sm.tmem_base);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  pdl_wait();  // global memory only after the previous kernel of the stream
  pdl_trigger();
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 320,
                 t_dq = tmem + 384;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_qkv);
      tma_prefetch_desc(&tm_dout);
      uint32_t qdo_it = 0;
      bool ok = true;
      int n = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
        int kt, h, b;
        bwd_decode(item, H * B, H, kt, h, b);
        const int kb = n & 1;
        if (!(ok = mbar_wait_bounded(&sm.kv_empty[kb], ((n >> 1) & 1) ^ 1, abort_flag, err,
                                     limit)))
          break;
        mbar_arrive_expect_tx(&sm.kv_full[kb], 2 * kTileBytes);
        tma_load_3d(sm.k[kb], &tm_qkv, &sm.kv_full[kb], C + h * kD, kt * kTile, b);
        tma_load_3d(sm.v[kb], &tm_qkv, &sm.kv_full[kb], 2 * C + h * kD, kt * kTile, b);
        for (int i = first_q(kt); i < n_t; ++i, ++qdo_it) {
          const int st = qdo_it & 1;
          if (!(ok = mbar_wait_bounded(&sm.qdo_empty[st], ((qdo_it >> 1) & 1) ^ 1, abort_flag, err,
                                       limit)))
            break;
          mbar_arrive_expect_tx(&sm.qdo_full[st], 2 * kTileBytes);
          tma_load_3d(sm.q[st], &tm_qkv, &sm.qdo_full[st], h * kD, i * kTile, b);
          tma_load_3d(sm.dout[st], &tm_dout, &sm.qdo_full[st], h * kD, i * kTile, b);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc_kq = make_idesc_bf16(128, 128, 0, 0);  // M=keys, N=queries
      constexpr uint32_t idesc_kd = make_idesc_bf16(128, kD, 0, 1);   // M=keys, N=D, B MN-major
      constexpr uint32_t idesc_qd = make_idesc_bf16(128, kD, 1, 1);   // M=queries, N=D, A,B MN-major
      const uint32_t p_addr = smem_u32(sm.p), ds_addr = smem_u32(sm.ds);
      uint32_t qdo_it = 0, t = 0;
      bool ok = true, issued = false;
      int n = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
        int kt, h, b;
        bwd_decode(item, H * B, H, kt, h, b);
        const int kb = n & 1;
        const uint32_t k_addr = smem_u32(sm.k[kb]), v_addr = smem_u32(sm.v[kb]);
        if (!(ok = mbar_wait_bounded(&sm.kv_full[kb], (n >> 1) & 1, abort_flag, err, limit))) break;
        int it = 0;
        for (int i = first_q(kt); i < n_t; ++i, ++it, ++qdo_it, ++t) {
          const int st = qdo_it & 1;
          if (!(ok = mbar_wait_bounded(&sm.qdo_full[st], (qdo_it >> 1) & 1, abort_flag, err,
                                       limit)))
            break;
          if (!(ok = mbar_wait_bounded(&sm.s_free, (t & 1) ^ 1, abort_flag, err, limit))) break;
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sm.q[st]), do_addr = smem_u32(sm.dout[st]);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            umma_bf16(t_s, make_sdesc_sw128(k_addr + kk * 32, 16, 1024),
                      make_sdesc_sw128(q_addr + kk * 32, 16, 1024), idesc_kq, kk > 0);
            umma_bf16(t_dp, make_sdesc_sw128(v_addr + kk * 32, 16, 1024),
                      make_sdesc_sw128(do_addr + kk * 32, 16, 1024), idesc_kq, kk > 0);
          }
          issued = true;
          umma_commit(&sm.s_full);
          if (!(ok = mbar_wait_bounded(&sm.p_ready, t & 1, abort_flag, err, limit))) break;
          // dV/dK of the previous item read out: waited only here, so this
          // item's first S^T / dP^T overlap that read-out
          if (it == 0 &&
              !(ok = mbar_wait_bounded(&sm.dkv_free, (n & 1) ^ 1, abort_flag, err, limit)))
            break;
          tc_fence_after();
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
          if (!(ok = mbar_wait_bounded(&sm.dq_free, (t & 1) ^ 1, abort_flag, err, limit))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk)
            umma_bf16(t_dq, make_sdesc_sw128(ds_addr + kk * 2048, kTileBytes, 1024),
                      make_sdesc_sw128(k_addr + kk * 2048, kTileBytes, 1024), idesc_qd, kk > 0);
          umma_commit(&sm.dq_full);
          umma_commit(&sm.pds_free);
          umma_commit(&sm.qdo_empty[st]);
        }
        if (!ok) break;
        umma_commit(&sm.kv_empty[n & 1]);
        umma_commit(&sm.dkv_full);
      }
      if (!ok && issued) {
        umma_commit(&sm.drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&sm.drain, 0) && global_timer_ns() - t0 < 100000000ull) {
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ compute warps
    const int wi = warp - 2;
    const int q4 = warp & 3;
    const int hh = wi >> 2;        // query half of each tile
    const int r = q4 * 32 + lane;  // key row within the tile (and query row for dQ)
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float sl2 = scale * kLog2e;
    const uint64_t sl2x2 = f2_splat(sl2);
    float* st_lse = sm.stat[wi][0];
    float* st_dl = sm.stat[wi][1];
    uint32_t t = 0;
    bool ok = true;
    int n = 0;
    int dq_pending_q0 = -1, dq_pending_b = 0, dq_pending_h = 0;
    // read out dQ of the previous tile (TMEM lanes = its queries) into dq_acc
    auto flush_dq = [&]() -> bool {
      if (dq_pending_q0 < 0) return true;
      const bool w = mbar_wait_bounded(&sm.dq_full, (t - 1) & 1, abort_flag, err, limit);
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
      uint32_t raw[32];
      tmem_ld_32cols(t_dq + lane_off + (uint32_t)(hh * 32), raw);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.dq_free);
      const int qi = dq_pending_q0 + r;
      if (qi < S) {
        float* dqrow = dq_acc + ((size_t)dq_pending_b * S + qi) * C + dq_pending_h * kD + hh * 32;
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          red_add_v4(dqrow + i, __uint_as_float(raw[i]), __uint_as_float(raw[i + 1]),
                     __uint_as_float(raw[i + 2]), __uint_as_float(raw[i + 3]));
      }
      dq_pending_q0 = -1;
      return true;
    };
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
      int kt, h, b;
      bwd_decode(item, H * B, H, kt, h, b);
      const int kj = kt * kTile + r;
      const bool key_ok = kj < S && !(key_pad && __ldg(key_pad + (size_t)b * S + kj) != 0);
      for (int i = first_q(kt); i < n_t; ++i, ++t) {
        const int q0 = i * kTile;
        const int qc0 = q0 + hh * 64;  // first query of this warp's half
        // this warp's 64 query statistics -> shared memory (queries >= S: p = 0)
        {
          const float* lrow = lse2 + ((size_t)b * H + h) * S;
          const float* drow = delta + ((size_t)b * H + h) * S;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int qi = qc0 + u * 32 + lane;
            // stored negated, so that P^T and dS^T take packed FMAs/adds
            st_lse[u * 32 + lane] = qi < S ? -__ldg(lrow + qi) : -INFINITY;
            st_dl[u * 32 + lane] = qi < S ? -__ldg(drow + qi) : 0.f;
          }
          __syncwarp();
        }
        ok = mbar_wait_bounded(&sm.s_full, t & 1, abort_flag, err, limit);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        // the previous tile's MMAs must be done reading P^T / dS^T
        ok = mbar_wait_bounded(&sm.pds_free, (t & 1) ^ 1, abort_flag, err, limit);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        const bool diag = causal && (qc0 < kt * kTile + kTile);  // some query < some key
        uint8_t* pb = sm.p + hh * kTileBytes;
        uint8_t* db = sm.ds + hh * kTileBytes;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {  // two 32-query chunks of this warp's half
          uint32_t rs[32], rdp[32];
          tmem_ld_32cols(t_s + lane_off + (uint32_t)(hh * 64 + cc * 32), rs);
          tmem_ld_32cols(t_dp + lane_off + (uint32_t)(hh * 64 + cc * 32), rdp);
          tmem_ld_wait();
          float p[32], ds[32];
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4) {
            const float4 l4 = *reinterpret_cast<const float4*>(st_lse + cc * 32 + 4 * c4);
            const float4 d4 = *reinterpret_cast<const float4*>(st_dl + cc * 32 + 4 * c4);
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
            const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
            for (int u = 0; u < 4; u += 2) {
              const int c = 4 * c4 + u;
              float a0, a1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), sl2x2,
                               f2_pack(lv[u], lv[u + 1])),
                        a0, a1);
              const bool v0 = key_ok && (!diag || kj <= qc0 + cc * 32 + c);
              const bool v1 = key_ok && (!diag || kj <= qc0 + cc * 32 + c + 1);
              p[c] = v0 ? ex2_approx(a0) : 0.f;
              p[c + 1] = v1 ? ex2_approx(a1) : 0.f;
              const uint64_t dd = f2_add(
                  f2_pack(__uint_as_float(rdp[c]), __uint_as_float(rdp[c + 1])),
                  f2_pack(dv[u], dv[u + 1]));
              f2_unpack(f2_mul(f2_pack(p[c], p[c + 1]), dd), ds[c], ds[c + 1]);
            }
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w, v;
            w.x = pack_bf16x2(p[8 * q + 0], p[8 * q + 1]);
            w.y = pack_bf16x2(p[8 * q + 2], p[8 * q + 3]);
            w.z = pack_bf16x2(p[8 * q + 4], p[8 * q + 5]);
            w.w = pack_bf16x2(p[8 * q + 6], p[8 * q + 7]);
            v.x = pack_bf16x2(ds[8 * q + 0], ds[8 * q + 1]);
            v.y = pack_bf16x2(ds[8 * q + 2], ds[8 * q + 3]);
            v.z = pack_bf16x2(ds[8 * q + 4], ds[8 * q + 5]);
            v.w = pack_bf16x2(ds[8 * q + 6], ds[8 * q + 7]);
            st_sw128_chunk(pb, r, cc * 4 + q, w);
            st_sw128_chunk(db, r, cc * 4 + q, v);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_free);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_ready);
        // dQ of the previous tile, then remember this one
        if (!flush_dq()) { ok = false; break; }
        dq_pending_q0 = q0;
        dq_pending_b = b;
        dq_pending_h = h;
      }
      if (!ok) break;
      ok = flush_dq();  // the last tile of this item (t was already advanced past it)
      if (!ok) break;
      // dK, dV of this key tile (thread = key row, 32 of the 64 columns)
      ok = mbar_wait_bounded(&sm.dkv_full, n & 1, abort_flag, err, limit);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      uint32_t rk[32], rv[32];
      tmem_ld_32cols(t_dk + lane_off + (uint32_t)(hh * 32), rk);
      tmem_ld_32cols(t_dv + lane_off + (uint32_t)(hh * 32), rv);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.dkv_free);
      if (dbias) {
        // K and V bias gradients: column sums of this warp's 32 key rows x 32
        // columns (rows past S hold zeros), one atomic per column and warp
        float ck[32], cv[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          ck[c] = kj < S ? __uint_as_float(rk[c]) * scale : 0.f;
          cv[c] = kj < S ? __uint_as_float(rv[c]) : 0.f;
        }
        const float sk = chunk_column_sum(ck, lane);
        const float sv = chunk_column_sum(cv, lane);
        atomicAdd(dbias + C + h * kD + hh * 32 + lane, sk);
        atomicAdd(dbias + 2 * C + h * kD + hh * 32 + lane, sv);
      }
      if (kj < S) {
        __nv_bfloat16* krow = dqkv + ((size_t)b * S + kj) * 3 * C + C + h * kD + hh * 32;
        __nv_bfloat16* vrow = krow + C;
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
          reinterpret_cast<uint4*>(krow)[q] = wk;
          reinterpret_cast<uint4*>(vrow)[q] = wv;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

// ============================================================== backward, one (batch, head) per item
// For sequences of at most two 128-row tiles (S <= 256, the LM benchmark's
// shape) a work item is a whole (batch, head): the CTA walks its key tiles
// and, per key tile, the query tiles that see them. dQ of both query tiles
// then accumulates in TMEM across the key tiles (two 64-column buffers), so
// dQ leaves the kernel as bf16 written once: no f32 accumulator to zero, no
// red.add traffic and no conversion pass. TMEM: S^T 0, dP^T 128, dV 256,
// dK 320, dQ of query tile 0 / 1 at 384 / 448 (all 512 columns).
//
// Warps and per-step math are those of flash_bwd_kernel. Read-outs are
// deferred by one step: after producing P^T / dS^T of step i, the compute
// warps read out what step i - 1 completed (dQ of a query tile after its last
// key tile, dK / dV after a key tile's last query tile), so the tensor cores
// run step i while the results of step i - 1 leave.
struct BwdBhSmem {
  uint8_t k[2][kTileBytes];  // K/V by key-tile parity (the next tile loads early)
  uint8_t v[2][kTileBytes];
  uint8_t q[2][kTileBytes];
  uint8_t dout[2][kTileBytes];
  uint8_t p[2 * kTileBytes];   // P^T: 128 keys x 128 queries (two 64-query SW128 blocks)
  uint8_t ds[2 * kTileBytes];  // dS^T, same layout
  float stat[kBwdWarps][2][64];
  uint64_t kv_full[2], kv_empty[2];
  uint64_t qdo_full[2], qdo_empty[2];
  uint64_t s_full, s_free, p_ready, pds_free, dkv_full, dkv_free;
  uint64_t dq_full[2], dq_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};

__global__ void __launch_bounds__(kBwdThreads, 1)
    flash_bwd_bh_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                        const __grid_constant__ CUtensorMap tm_dout, const float* __restrict__ lse2,
                        const float* __restrict__ delta, __nv_bfloat16* __restrict__ dqkv,
                        const uint8_t* __restrict__ key_pad, int B, int S, int H, int causal,
                        float scale, float* __restrict__ dbias, uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  BwdBhSmem& sm = *reinterpret_cast<BwdBhSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int C = H * kD;
  const int n_t = (S + kTile - 1) / kTile;  // 1 or 2
  const int n_items = H * B;
  const uint64_t limit = g_fa_wait_limit_ns;
  volatile uint32_t* abort_flag = &sm.abort;
  auto first_q = [&](int kt) { return causal ? kt : 0; };
  // the last key tile that contributes to query tile qt
  auto last_k = [&](int qt) { return causal ? qt : n_t - 1; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
      mbar_init(&sm.qdo_full[i], 1);
      mbar_init(&sm.qdo_empty[i], 1);
      mbar_init(&sm.dq_full[i], 1);
      mbar_init(&sm.dq_free[i], kBwdWarps);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, kBwdWarps);
    mbar_init(&sm.p_ready, kBwdWarps);
    mbar_init(&sm.pds_free, 1);
    mbar_init(&sm.dkv_full, 1);
    mbar_init(&sm.dkv_free, kBwdWarps);
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<512>(&sm.tmem_base);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  pdl_wait();  // global memory only after the previous kernel of the stream
  pdl_trigger();
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 320,
                 t_dq = tmem + 384;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_qkv);
      tma_prefetch_desc(&tm_dout);
      uint32_t kv_it = 0, qdo_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const int h = item % H, b = item / H;
        for (int kt = 0; kt < n_t && ok; ++kt, ++kv_it) {
          const int kb = kv_it & 1;
          if (!(ok = mbar_wait_bounded(&sm.kv_empty[kb], ((kv_it >> 1) & 1) ^ 1, abort_flag, err,
                                       limit)))
            break;
          mbar_arrive_expect_tx(&sm.kv_full[kb], 2 * kTileBytes);
          tma_load_3d(sm.k[kb], &tm_qkv, &sm.kv_full[kb], C + h * kD, kt * kTile, b);
          tma_load_3d(sm.v[kb], &tm_qkv, &sm.kv_full[kb], 2 * C + h * kD, kt * kTile, b);
          for (int i = first_q(kt); i < n_t; ++i, ++qdo_it) {
            const int st = qdo_it & 1;
            if (!(ok = mbar_wait_bounded(&sm.qdo_empty[st], ((qdo_it >> 1) & 1) ^ 1, abort_flag,
                                         err, limit)))
              break;
            mbar_arrive_expect_tx(&sm.qdo_full[st], 2 * kTileBytes);
            tma_load_3d(sm.q[st], &tm_qkv, &sm.qdo_full[st], h * kD, i * kTile, b);
            tma_load_3d(sm.dout[st], &tm_dout, &sm.qdo_full[st], h * kD, i * kTile, b);
          }
        }
      }
    }
    __syncwarp();  // reconverge before the CTA-wide barrier at the end
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc_kq = make_idesc_bf16(128, 128, 0, 0);  // M=keys, N=queries
      constexpr uint32_t idesc_kd = make_idesc_bf16(128, kD, 0, 1);   // M=keys, N=D, B MN-major
      constexpr uint32_t idesc_qd = make_idesc_bf16(128, kD, 1, 1);   // M=queries, N=D
      const uint32_t p_addr = smem_u32(sm.p), ds_addr = smem_u32(sm.ds);
      uint32_t kv_it = 0, qdo_it = 0, t = 0;
      bool ok = true, issued = false;
      int n = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
        for (int kt = 0; kt < n_t && ok; ++kt, ++kv_it) {
          const int kb = kv_it & 1;
          const uint32_t k_addr = smem_u32(sm.k[kb]), v_addr = smem_u32(sm.v[kb]);
          if (!(ok = mbar_wait_bounded(&sm.kv_full[kb], (kv_it >> 1) & 1, abort_flag, err, limit)))
            break;
          int it = 0;
          for (int i = first_q(kt); i < n_t; ++i, ++it, ++qdo_it, ++t) {
            const int st = qdo_it & 1;
            if (!(ok = mbar_wait_bounded(&sm.qdo_full[st], (qdo_it >> 1) & 1, abort_flag, err,
                                         limit)))
              break;
            if (!(ok = mbar_wait_bounded(&sm.s_free, (t & 1) ^ 1, abort_flag, err, limit))) break;
            tc_fence_after();
            const uint32_t q_addr = smem_u32(sm.q[st]), do_addr = smem_u32(sm.dout[st]);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              umma_bf16(t_s, make_sdesc_sw128(k_addr + kk * 32, 16, 1024),
                        make_sdesc_sw128(q_addr + kk * 32, 16, 1024), idesc_kq, kk > 0);
              umma_bf16(t_dp, make_sdesc_sw128(v_addr + kk * 32, 16, 1024),
                        make_sdesc_sw128(do_addr + kk * 32, 16, 1024), idesc_kq, kk > 0);
            }
            issued = true;
            umma_commit(&sm.s_full);
            if (!(ok = mbar_wait_bounded(&sm.p_ready, t & 1, abort_flag, err, limit))) break;
            // dV/dK of the previous key tile read out (deferred by one step)
            if (it == 0 &&
                !(ok = mbar_wait_bounded(&sm.dkv_free, (kv_it & 1) ^ 1, abort_flag, err, limit)))
              break;
            tc_fence_after();
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
            // dQ of query tile i: first touched at key tile 0 in this item,
            // whose buffer the read-out of the previous item must have freed
            if (kt == 0 &&
                !(ok = mbar_wait_bounded(&sm.dq_free[i], (n & 1) ^ 1, abort_flag, err, limit)))
              break;
            tc_fence_after();
            const uint32_t t_dqi = t_dq + (uint32_t)(i * kD);
#pragma unroll
            for (int kk = 0; kk < kTile / 16; ++kk)
              umma_bf16(t_dqi, make_sdesc_sw128(ds_addr + kk * 2048, kTileBytes, 1024),
                        make_sdesc_sw128(k_addr + kk * 2048, kTileBytes, 1024), idesc_qd,
                        (kt > 0 || kk > 0));
            umma_commit(&sm.pds_free);
            umma_commit(&sm.qdo_empty[st]);
            if (kt == last_k(i)) umma_commit(&sm.dq_full[i]);
          }
          if (!ok) break;
          umma_commit(&sm.kv_empty[kb]);
          umma_commit(&sm.dkv_full);
        }
      }
      if (!ok && issued) {
        umma_commit(&sm.drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&sm.drain, 0) && global_timer_ns() - t0 < 100000000ull) {
        }
      }
    }
    __syncwarp();  // reconverge before the CTA-wide barrier at the end
  } else {
    // ------------------------------------------------------------ compute warps
    const int wi = warp - 2;
    const int q4 = warp & 3;
    const int hh = wi >> 2;        // query half of each tile (dims half of dQ/dK/dV)
    const int r = q4 * 32 + lane;  // key row of the tile (query row for dQ)
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float sl2 = scale * kLog2e;
    const uint64_t sl2x2 = f2_splat(sl2);
    float* st_lse = sm.stat[wi][0];
    float* st_dl = sm.stat[wi][1];
    uint32_t t = 0, kv_done = 0;
    bool ok = true;
    int n = 0;
    // read-outs completed by the previous step, done after the next step's P^T / dS^T
    struct Pending {
      int dq_tile = -1, dq_b = 0, dq_h = 0, dq_n = 0;
      int kv_tile = -1, kv_b = 0, kv_h = 0;
    } pend;
    auto readout_dq = [&](int qt, int b, int h, int nn) -> bool {
      const bool w = mbar_wait_bounded(&sm.dq_full[qt], nn & 1, abort_flag, err, limit);
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
      uint32_t raw[32];
      tmem_ld_32cols(t_dq + (uint32_t)(qt * kD) + lane_off + (uint32_t)(hh * 32), raw);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.dq_free[qt]);
      const int qi = qt * kTile + r;
      float vq[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) vq[c] = qi < S ? __uint_as_float(raw[c]) * scale : 0.f;
      if (dbias) {
        const float sq = chunk_column_sum(vq, lane);
        atomicAdd(dbias + h * kD + hh * 32 + lane, sq);
      }
      if (qi < S) {
        uint4* qrow = reinterpret_cast<uint4*>(dqkv + ((size_t)b * S + qi) * 3 * C + h * kD +
                                               hh * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(vq[8 * q + 0], vq[8 * q + 1]);
          w.y = pack_bf16x2(vq[8 * q + 2], vq[8 * q + 3]);
          w.z = pack_bf16x2(vq[8 * q + 4], vq[8 * q + 5]);
          w.w = pack_bf16x2(vq[8 * q + 6], vq[8 * q + 7]);
          qrow[q] = w;
        }
      }
      return true;
    };
    auto readout_dkv = [&](int kt, int b, int h) -> bool {
      const bool w = mbar_wait_bounded(&sm.dkv_full, kv_done & 1, abort_flag, err, limit);
      ++kv_done;
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
      uint32_t rk[32], rv[32];
      tmem_ld_32cols(t_dk + lane_off + (uint32_t)(hh * 32), rk);
      tmem_ld_32cols(t_dv + lane_off + (uint32_t)(hh * 32), rv);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.dkv_free);
      const int kj = kt * kTile + r;
      float ck[32], cv[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        ck[c] = kj < S ? __uint_as_float(rk[c]) * scale : 0.f;
        cv[c] = kj < S ? __uint_as_float(rv[c]) : 0.f;
      }
      if (dbias) {
        const float sk = chunk_column_sum(ck, lane);
        const float sv = chunk_column_sum(cv, lane);
        atomicAdd(dbias + C + h * kD + hh * 32 + lane, sk);
        atomicAdd(dbias + 2 * C + h * kD + hh * 32 + lane, sv);
      }
      if (kj < S) {
        __nv_bfloat16* krow = dqkv + ((size_t)b * S + kj) * 3 * C + C + h * kD + hh * 32;
        __nv_bfloat16* vrow = krow + C;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 wk, wv;
          wk.x = pack_bf16x2(ck[8 * q + 0], ck[8 * q + 1]);
          wk.y = pack_bf16x2(ck[8 * q + 2], ck[8 * q + 3]);
          wk.z = pack_bf16x2(ck[8 * q + 4], ck[8 * q + 5]);
          wk.w = pack_bf16x2(ck[8 * q + 6], ck[8 * q + 7]);
          wv.x = pack_bf16x2(cv[8 * q + 0], cv[8 * q + 1]);
          wv.y = pack_bf16x2(cv[8 * q + 2], cv[8 * q + 3]);
          wv.z = pack_bf16x2(cv[8 * q + 4], cv[8 * q + 5]);
          wv.w = pack_bf16x2(cv[8 * q + 6], cv[8 * q + 7]);
          reinterpret_cast<uint4*>(krow)[q] = wk;
          reinterpret_cast<uint4*>(vrow)[q] = wv;
        }
      }
      return true;
    };
    auto flush = [&]() -> bool {
      bool good = true;
      if (pend.dq_tile >= 0) good = readout_dq(pend.dq_tile, pend.dq_b, pend.dq_h, pend.dq_n);
      pend.dq_tile = -1;
      if (good && pend.kv_tile >= 0) good = readout_dkv(pend.kv_tile, pend.kv_b, pend.kv_h);
      pend.kv_tile = -1;
      return good;
    };
    // softmax statistics of this warp's queries (both query tiles, negated
    // for the packed FMAs), loaded one item ahead so their latency hides
    // behind the previous item's steps
    float cl[2][2], cd[2][2], nl[2][2], nd[2][2];
    auto load_stats = [&](int item, float (&l)[2][2], float (&d)[2][2]) {
      const int h = item % H, b = item / H;
      const float* lrow = lse2 + ((size_t)b * H + h) * S;
      const float* drow = delta + ((size_t)b * H + h) * S;
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int qi = i * kTile + hh * 64 + u * 32 + lane;
          const bool in = i < n_t && qi < S;
          l[i][u] = in ? -__ldg(lrow + qi) : -INFINITY;
          d[i][u] = in ? -__ldg(drow + qi) : 0.f;
        }
    };
    if (blockIdx.x < n_items) load_stats(blockIdx.x, cl, cd);
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
      const int h = item % H, b = item / H;
      if (item + (int)gridDim.x < n_items) load_stats(item + gridDim.x, nl, nd);
      for (int kt = 0; kt < n_t && ok; ++kt) {
        const int kj = kt * kTile + r;
        const bool key_ok = kj < S && !(key_pad && __ldg(key_pad + (size_t)b * S + kj) != 0);
        for (int i = first_q(kt); i < n_t; ++i, ++t) {
          const int q0 = i * kTile;
          const int qc0 = q0 + hh * 64;  // first query of this warp's half
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            st_lse[u * 32 + lane] = i == 0 ? cl[0][u] : cl[1][u];
            st_dl[u * 32 + lane] = i == 0 ? cd[0][u] : cd[1][u];
          }
          __syncwarp();
          ok = mbar_wait_bounded(&sm.s_full, t & 1, abort_flag, err, limit);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          ok = mbar_wait_bounded(&sm.pds_free, (t & 1) ^ 1, abort_flag, err, limit);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          tc_fence_after();
          const bool diag = causal && (qc0 < kt * kTile + kTile);
          uint8_t* pb = sm.p + hh * kTileBytes;
          uint8_t* db = sm.ds + hh * kTileBytes;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            uint32_t rs[32], rdp[32];
            tmem_ld_32cols(t_s + lane_off + (uint32_t)(hh * 64 + cc * 32), rs);
            tmem_ld_32cols(t_dp + lane_off + (uint32_t)(hh * 64 + cc * 32), rdp);
            tmem_ld_wait();
            float p[32], ds[32];
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const float4 l4 = *reinterpret_cast<const float4*>(st_lse + cc * 32 + 4 * c4);
              const float4 d4 = *reinterpret_cast<const float4*>(st_dl + cc * 32 + 4 * c4);
              const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
              const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
              for (int u = 0; u < 4; u += 2) {
                const int c = 4 * c4 + u;
                float a0, a1;
                f2_unpack(f2_fma(f2_pack(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])),
                                 sl2x2, f2_pack(lv[u], lv[u + 1])),
                          a0, a1);
                const bool v0 = key_ok && (!diag || kj <= qc0 + cc * 32 + c);
                const bool v1 = key_ok && (!diag || kj <= qc0 + cc * 32 + c + 1);
                p[c] = v0 ? ex2_approx(a0) : 0.f;
                p[c + 1] = v1 ? ex2_approx(a1) : 0.f;
                const uint64_t dd = f2_add(
                    f2_pack(__uint_as_float(rdp[c]), __uint_as_float(rdp[c + 1])),
                    f2_pack(dv[u], dv[u + 1]));
                f2_unpack(f2_mul(f2_pack(p[c], p[c + 1]), dd), ds[c], ds[c + 1]);
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w, v;
              w.x = pack_bf16x2(p[8 * q + 0], p[8 * q + 1]);
              w.y = pack_bf16x2(p[8 * q + 2], p[8 * q + 3]);
              w.z = pack_bf16x2(p[8 * q + 4], p[8 * q + 5]);
              w.w = pack_bf16x2(p[8 * q + 6], p[8 * q + 7]);
              v.x = pack_bf16x2(ds[8 * q + 0], ds[8 * q + 1]);
              v.y = pack_bf16x2(ds[8 * q + 2], ds[8 * q + 3]);
              v.z = pack_bf16x2(ds[8 * q + 4], ds[8 * q + 5]);
              v.w = pack_bf16x2(ds[8 * q + 6], ds[8 * q + 7]);
              st_sw128_chunk(pb, r, cc * 4 + q, w);
              st_sw128_chunk(db, r, cc * 4 + q, v);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.s_free);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.p_ready);
          // results of the previous step, then queue this step's
          if (!flush()) { ok = false; break; }
          if (kt == last_k(i)) {
            pend.dq_tile = i;
            pend.dq_b = b;
            pend.dq_h = h;
            pend.dq_n = n;
          }
          if (i == n_t - 1) {
            pend.kv_tile = kt;
            pend.kv_b = b;
            pend.kv_h = h;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          cl[i][u] = nl[i][u];
          cd[i][u] = nd[i][u];
        }
    }
    if (ok) flush();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

}  // namespace


void set_flash_wait_limit_ns(uint64_t ns) {
  cudaMemcpyToSymbol(g_fa_wait_limit_ns, &ns, sizeof(ns));
}

// FLODL_FLASH_FWD=v1 selects the one-CTA-per-SM forward (8 softmax warps, P
// in shared memory) instead of the two-CTA-per-SM kernel with P in TMEM.
static bool use_fwd_v1() {
  static const bool v1 = [] {
    const char* e = std::getenv("FLODL_FLASH_FWD");
    return e != nullptr && std::strcmp(e, "v1") == 0;
  }();
  return v1;
}

static cudaError_t launch_flash_fwd2(const FlashArgs& a, const CUtensorMap& tm, cudaStream_t st) {
  const int smem = (int)sizeof(Fwd2Smem) + 1024;
  static std::atomic<uint64_t> done{0};
  static std::atomic<int> per_sm{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load(std::memory_order_relaxed) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(flash_fwd2_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    // the largest shared-memory carveout, so that two CTAs fit on an SM
    e = cudaFuncSetAttribute(flash_fwd2_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    // CTAs per SM from the shared memory and register budgets (the runtime's
    // occupancy query answered 1 here although two fit)
    int smem_sm = 0, reserved = 0, regs_sm = 0;
    cudaFuncAttributes fa{};
    if (cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) !=
            cudaSuccess ||
        cudaFuncGetAttributes(&fa, flash_fwd2_kernel) != cudaSuccess)
      return cudaGetLastError();
    const int by_smem = smem_sm / (smem + reserved);
    const int regs_cta = ((fa.numRegs + 7) / 8 * 8) * kF2Threads;
    const int by_regs = regs_cta > 0 ? regs_sm / regs_cta : 1;
    per_sm.store(std::max(1, std::min(2, std::min(by_smem, by_regs))));
    done.fetch_or(bit);
  }
  const int64_t items = (int64_t)((a.S + kTile - 1) / kTile) * a.H * a.B;
  const int grid = (int)std::min<int64_t>(items, (int64_t)num_sms() * per_sm.load());
  cudaError_t le = launch_pdl(flash_fwd2_kernel, dim3(grid), dim3(kF2Threads), smem, st, tm, a.out,
                              a.lse2, a.key_pad, a.B, a.S, a.H, a.causal ? 1 : 0, a.scale,
                              a.err ? a.err : default_err_word());
  if (le != cudaSuccess) return le;
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_flash_fwd(const FlashArgs& a, cudaStream_t st) {
  if (a.D != kD || a.S <= 0 || a.B <= 0 || a.H <= 0) return cudaErrorInvalidValue;
  CUtensorMap tm;
  if (!make_map_3d(&tm, a.qkv, a.B, a.S, 3 * a.H * kD)) return cudaErrorInvalidValue;
  if (!use_fwd_v1()) return launch_flash_fwd2(a, tm, st);
  const int smem = (int)sizeof(FwdSmem) + 1024;
  {
    // the dynamic shared-memory opt-in is a per-device function attribute
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done.load(std::memory_order_relaxed) & bit)) {
      cudaError_t e = cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      done.fetch_or(bit);
    }
  }
  const int64_t items = (int64_t)((a.S + kTile - 1) / kTile) * a.H * a.B;
  const int grid = (int)std::min<int64_t>(items, (int64_t)num_sms());
  flash_fwd_kernel<<<grid, kFwdThreads, smem, st>>>(tm, a.out, a.lse2, a.key_pad, a.B, a.S, a.H,
                                                     a.causal ? 1 : 0, a.scale,
                                                     a.err ? a.err : default_err_word());
  note_launch();
  return cudaGetLastError();
}

// FLODL_FLASH_BWD=v1 keeps the key-tile kernel (f32 dQ accumulator) for
// every sequence length instead of the per-(batch, head) kernel for S <= 256.
static bool use_bwd_v1() {
  static const bool v1 = [] {
    const char* e = std::getenv("FLODL_FLASH_BWD");
    return e != nullptr && std::strcmp(e, "v1") == 0;
  }();
  return v1;
}

bool flash_bwd_needs_dq_acc(int S) { return S > 2 * kTile || use_bwd_v1(); }

cudaError_t launch_flash_bwd(const FlashArgs& a, cudaStream_t st) {
  if (a.D != kD || a.S <= 0 || a.B <= 0 || a.H <= 0) return cudaErrorInvalidValue;
  const int C = a.H * kD;
  CUtensorMap tm_qkv, tm_do;
  if (!make_map_3d(&tm_qkv, a.qkv, a.B, a.S, 3 * C)) return cudaErrorInvalidValue;
  if (!make_map_3d(&tm_do, a.dout, a.B, a.S, C)) return cudaErrorInvalidValue;
  const int64_t rows = (int64_t)a.B * a.S * a.H;
  if (rows >= (int64_t)1 << 31) return cudaErrorInvalidValue;  // 32-bit row indices
  int pre_blocks = (int)std::min<int64_t>((rows + 31) / 32, (int64_t)num_sms() * 16);
  if (!flash_bwd_needs_dq_acc(a.S)) {
    // dQ stays in TMEM: delta only, then one kernel per (batch, head)
    cudaError_t le = launch_pdl(flash_bwd_pre_kernel, dim3(pre_blocks), dim3(256), 0, st, a.dout,
                                a.out, a.delta, (float*)nullptr, a.B, a.S, a.H);
    if (le != cudaSuccess) return le;
    const int smem = (int)sizeof(BwdBhSmem) + 1024;
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done.load(std::memory_order_relaxed) & bit)) {
      cudaError_t e = cudaFuncSetAttribute(flash_bwd_bh_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      done.fetch_or(bit);
    }
    const int grid = std::min(a.B * a.H, num_sms());
    le = launch_pdl(flash_bwd_bh_kernel, dim3(grid), dim3(kBwdThreads), smem, st, tm_qkv, tm_do,
                    (const float*)a.lse2, (const float*)a.delta, a.dqkv, a.key_pad, a.B, a.S,
                    a.H, a.causal ? 1 : 0, a.scale, a.dbias, a.err ? a.err : default_err_word());
    if (le != cudaSuccess) return le;
    note_launch(2);
    return cudaGetLastError();
  }
  if (a.dq_acc == nullptr) return cudaErrorInvalidValue;
  flash_bwd_pre_kernel<<<pre_blocks, 256, 0, st>>>(a.dout, a.out, a.delta, a.dq_acc, a.B, a.S, a.H);
  const int smem = (int)sizeof(BwdSmem) + 1024;
  {
    // the dynamic shared-memory opt-in is a per-device function attribute
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done.load(std::memory_order_relaxed) & bit)) {
      cudaError_t e = cudaFuncSetAttribute(flash_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      done.fetch_or(bit);
    }
  }
  const int64_t items = (int64_t)((a.S + kTile - 1) / kTile) * a.H * a.B;
  const int grid = (int)std::min<int64_t>(items, (int64_t)num_sms());
  flash_bwd_kernel<<<grid, kBwdThreads, smem, st>>>(tm_qkv, tm_do, a.lse2, a.delta, a.dq_acc, a.dqkv,
                                            a.key_pad, a.B, a.S, a.H, a.causal ? 1 : 0, a.scale,
                                            a.dbias, a.err ? a.err : default_err_word());
  const int T = a.B * a.S;
  const int groups = C / 8;  // dQ column groups
  const int gw = std::min(kPostMaxThreads, (groups + 31) / 32 * 32);  // threads per row lane
  const int gy = (groups + gw - 1) / gw;
  const int lanes = kPostMaxThreads / gw;
  const int gx = std::max(1, std::min(T, num_sms() / gy));
  const int rpb = (T + gx - 1) / gx;
  flash_bwd_post_kernel<<<dim3(gx, gy), gw * lanes, 0, st>>>(a.dq_acc, a.dqkv, T, C, a.scale,
                                                            a.dbias, rpb, gw);
  note_launch(3);
  return cudaGetLastError();
}

}  // namespace flodl
