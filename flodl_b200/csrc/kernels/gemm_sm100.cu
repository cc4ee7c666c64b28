// Persistent warp-specialised bf16 GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA).
//
//   C[M,N] = epilogue( sum_k A[m,k] * B[n,k] )
//
// Operand storage (all bf16, row-major in memory):
//   A K-major : [M, K]   (activations x, upstream grads dY)
//   A MN-major: [K, M]   (dY viewed transposed for the weight gradient)
//   B K-major : [N, K]   (nn.Linear weight W[out,in])
//   B MN-major: [K, N]   (W used as [in,out] for the input gradient, x for wgrad)
//
// This one engine serves the three GEMMs of a Linear layer (the reference calls
// torch::linear / cuBLAS for these: flodl-sys/ops_training.cpp:400-414):
//   forward   y  = x  W^T       A=x  (K-major), B=W (K-major)
//   dgrad     dx = dy W         A=dy (K-major), B=W (MN-major)
//   wgrad     dW = dy^T x       A=dy (MN-major), B=x (MN-major), f32 accumulate
//
// Warp roles (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0   : TMA producer (one elected lane)
//   warp 1   : TMEM allocator + MMA issuer (one elected lane)
//   warps 2-5: epilogue (TMEM -> registers -> bias/GELU/residual -> global)
// Two TMEM accumulator buffers let the epilogue of tile i overlap the MMAs of
// tile i+1. No TMA multicast is used anywhere.
#include "sm100_ptx.cuh"
#include "gemm_sm100.h"

#include <cstdio>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace flodl {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kEpiWarps = 8;                      // two per SM sub-partition
constexpr int kThreads = 64 + 32 * kEpiWarps;     // producer + MMA + epilogue

__device__ uint64_t g_wait_limit_ns = 2000000000ull;  // 2 s

// Epilogue staging: each epilogue warp owns kSlots 4 KB slots of shared
// memory. A slot holds one 32x32 output chunk (f32, 128B swizzle) or one bf16
// output chunk plus one bf16 GELU' chunk (2 KB each, 64B swizzle). Chunks
// leave through TMA stores (full, coalesced lines). Epilogues with an input
// (residual, GELU' operand) take two slots: the input of chunk j+1 arrives by
// TMA into the other slot while chunk j is computed. Epilogues without one
// take a single slot (the store of chunk j-1 reads it while chunk j is
// computed), which leaves shared memory for one more operand stage.
constexpr int kSlotBytes = 4096;

// kPair: a CTA pair computes a 256 x BN tile with one cta_group::2 MMA; each
// CTA stages 128 rows of A and BN/2 rows of B per K step.
template <int BN, int kSlots, bool kPair = false>
struct GemmCfg {
  static constexpr int kStagingBytes = kEpiWarps * kSlots * kSlotBytes;
  static constexpr int kATileBytes = kBM * kBK * 2;                      // 16 KB
  static constexpr int kBTileBytes = (kPair ? BN / 2 : BN) * kBK * 2;  // 32 or 16 KB
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  // as many operand stages as fit beside the staging slots (at most 8)
  static constexpr int kFit = (227 * 1024 - kStagingBytes - 1024 - 512) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  // double-buffered accumulator, allocated as a power of two (BN = 192: 512)
  static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;
  static_assert(BN % 64 == 0 && BN <= 256, "tile width");
  static constexpr int kSmemBytes =
      kStages * kStageBytes + kStagingBytes + 1024 /*align*/ + 512 /*barriers*/;
  static_assert(kStages <= 8, "barrier arrays");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
};

struct SmemCtl {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint64_t epi_in[kEpiWarps * 2];  // epilogue input loads, one per warp slot
  uint32_t tmem_base;
  uint32_t abort;
};
static_assert(sizeof(SmemCtl) <= 512, "barrier block");

__device__ __forceinline__ void epilogue_chunk(const GemmEpilogue& ep, int row, int col0,
                                               int M, int N, const uint32_t (&acc)[32]) {
  if (row >= M) return;
  float v[32];
  const float alpha = ep.alpha_ptr ? ep.alpha * __ldg(ep.alpha_ptr) : ep.alpha;
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(acc[i]) * alpha;

  const bool full_cols = (col0 + 32 <= N);
  if (ep.bias) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      int c = col0 + i;
      v[i] += (c < N) ? __ldg(ep.bias + c) : 0.f;
    }
  }
  if (ep.flags & kEpiGelu) {
    float dg[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) gelu_and_grad(v[i], v[i], dg[i]);
    if (ep.aux) {  // keep GELU' for the backward pass
      __nv_bfloat16* aux = reinterpret_cast<__nv_bfloat16*>(ep.aux) + (size_t)row * ep.ld_aux;
      if (full_cols && ((ep.ld_aux & 7) == 0)) {
        uint4* dst = reinterpret_cast<uint4*>(aux + col0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(dg[8 * q + 0], dg[8 * q + 1]);
          w.y = pack_bf16x2(dg[8 * q + 2], dg[8 * q + 3]);
          w.z = pack_bf16x2(dg[8 * q + 4], dg[8 * q + 5]);
          w.w = pack_bf16x2(dg[8 * q + 6], dg[8 * q + 7]);
          dst[q] = w;
        }
      } else {
        for (int i = 0; i < 32; ++i)
          if (col0 + i < N) aux[col0 + i] = __float2bfloat16_rn(dg[i]);
      }
    }
  }
  if (ep.flags & kEpiDGelu) {  // multiply by the stored GELU'
    const __nv_bfloat16* aux =
        reinterpret_cast<const __nv_bfloat16*>(ep.aux) + (size_t)row * ep.ld_aux;
    if (full_cols && ((ep.ld_aux & 7) == 0)) {
      const uint4* src = reinterpret_cast<const uint4*>(aux + col0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w = src[q];
        uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float2 f = unpack_bf16x2(ws[h]);
          v[8 * q + 2 * h + 0] *= f.x;
          v[8 * q + 2 * h + 1] *= f.y;
        }
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) v[i] *= __bfloat162float(aux[col0 + i]);
    }
  }
  if (ep.residual) {
    const float* res = ep.residual + (size_t)row * ep.ld_res;
    if (full_cols && ((ep.ld_res & 3) == 0)) {
      const float4* src = reinterpret_cast<const float4*>(res + col0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 r = src[q];
        v[4 * q + 0] += r.x;
        v[4 * q + 1] += r.y;
        v[4 * q + 2] += r.z;
        v[4 * q + 3] += r.w;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) v[i] += res[col0 + i];
    }
  }

  if (ep.out_f32) {
    float* out = reinterpret_cast<float*>(ep.out) + (size_t)row * ep.ld_out;
    if (full_cols && ((ep.ld_out & 3) == 0)) {
      if (ep.flags & kEpiAccumulate) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          red_add_v4(out + col0 + 4 * q, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      } else {
        float4* dst = reinterpret_cast<float4*>(out + col0);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    } else {
      for (int i = 0; i < 32; ++i) {
        int c = col0 + i;
        if (c >= N) break;
        if (ep.flags & kEpiAccumulate)
          atomicAdd(out + c, v[i]);
        else
          out[c] = v[i];
      }
    }
  } else {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(ep.out) + (size_t)row * ep.ld_out;
    if (full_cols && ((ep.ld_out & 7) == 0)) {
      uint4* dst = reinterpret_cast<uint4*>(out + col0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
        w.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
        w.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
        w.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
        dst[q] = w;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) out[col0 + i] = __float2bfloat16_rn(v[i]);
    }
  }
}

// What the epilogue prefetches (TMA) into a staging slot before a chunk's math.
enum EpiInput : int { kInNone = 0, kInResidual = 1, kInAux = 2 };

// TMA-store epilogue of one 32x32 chunk. The warp's staging slot (4 KB) holds
// the chunk in the layout its tensor maps use: f32 rows of 128 B with the
// 128-byte swizzle (chunk q of row r at q ^ (r & 7)), or bf16 rows of 64 B with
// the 64-byte swizzle (q ^ ((r >> 1) & 3)) at offset 0 plus, for a second bf16
// tensor (GELU' out, or the GELU' input), at offset 2048. Inputs
// (residual f32 / GELU' bf16) were brought in by TMA at the same
// positions the outputs use, so each lane reads and writes its own row only.
// Out-of-range rows/columns need no checks: TMA loads fill them with zeros and
// TMA stores clip them; only the bias needs a bound.
__device__ __forceinline__ void epilogue_chunk_tma(const GemmEpilogue& ep, float alpha,
                                                   const CUtensorMap* tmOut,
                                                   const CUtensorMap* tmAux, uint8_t* slot,
                                                   int row0, int col0, int lane, int N,
                                                   const uint32_t (&acc)[32], bool wait_slot,
                                                   float* cs_keep, float* cq_keep) {
  float v[32];
  if (ep.bias && col0 + 32 <= N && (reinterpret_cast<uintptr_t>(ep.bias) & 15) == 0) {
    // v = acc * alpha + bias, two columns per packed FMA
    const float4* b4 = reinterpret_cast<const float4*>(ep.bias + col0);
    const uint64_t al = f2_splat(alpha);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = __ldg(b4 + q);
      f2_unpack(f2_fma(f2_pack(__uint_as_float(acc[4 * q]), __uint_as_float(acc[4 * q + 1])), al,
                       f2_pack(b.x, b.y)),
                v[4 * q], v[4 * q + 1]);
      f2_unpack(f2_fma(f2_pack(__uint_as_float(acc[4 * q + 2]), __uint_as_float(acc[4 * q + 3])),
                       al, f2_pack(b.z, b.w)),
                v[4 * q + 2], v[4 * q + 3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(acc[i]) * alpha;
    if (ep.bias) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += (col0 + i < N) ? __ldg(ep.bias + col0 + i) : 0.f;
    }
  }
  const int sw64 = (lane >> 1) & 3;
  const int sw128 = lane & 7;
  const bool aux_out = (ep.flags & kEpiGelu) && ep.aux;
  // single-slot staging: the previous chunk's store must have read the slot
  // (it did so while this chunk's accumulator was read and its math ran)
  auto slot_free = [&]() {
    if (wait_slot) {
      if (lane == 0) bulk_wait_group_read<0>();
      __syncwarp();
    }
  };
  if (ep.flags & kEpiGelu) {
    float dg[32];
#pragma unroll
    for (int i = 0; i < 32; i += 2) gelu_and_grad2(v[i], v[i + 1], v[i], v[i + 1], dg[i], dg[i + 1]);
    slot_free();
    wait_slot = false;
    if (aux_out) {  // GELU', kept for the backward pass
      uint8_t* a = slot + 2048 + lane * 64;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(dg[8 * q + 0], dg[8 * q + 1]);
        w.y = pack_bf16x2(dg[8 * q + 2], dg[8 * q + 3]);
        w.z = pack_bf16x2(dg[8 * q + 4], dg[8 * q + 5]);
        w.w = pack_bf16x2(dg[8 * q + 6], dg[8 * q + 7]);
        *reinterpret_cast<uint4*>(a + ((q ^ sw64) * 16)) = w;
      }
    }
  }
  if (ep.flags & kEpiDGelu) {  // multiply by the stored GELU' (staged at +2048)
    const uint8_t* a = slot + 2048 + lane * 64;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = *reinterpret_cast<const uint4*>(a + ((q ^ sw64) * 16));
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16x2(ws[h]);
        f2_unpack(f2_mul(f2_pack(v[8 * q + 2 * h], v[8 * q + 2 * h + 1]), f2_pack(f.x, f.y)),
                  v[8 * q + 2 * h], v[8 * q + 2 * h + 1]);
      }
    }
  }
  // Column sums (bias gradient of the next layer; batch-norm statistics with
  // the squares): out-of-range rows hold zeros. With cs_keep / cq_keep the
  // chunk's sums are kept in the warp's registers (one column per lane) and
  // flushed once per CTA, else one atomic per column and chunk.
  if (ep.colsum) {
    const float s = chunk_column_sum(v, lane);
    if (cs_keep)
      *cs_keep += s;
    else if (col0 + lane < N)
      atomicAdd(ep.colsum + col0 + lane, s);
  }
  if (ep.colsumsq) {
    float sq[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) sq[i] = v[i] * v[i];
    const float s = chunk_column_sum(sq, lane);
    if (cq_keep)
      *cq_keep += s;
    else if (col0 + lane < N)
      atomicAdd(ep.colsumsq + col0 + lane, s);
  }
  slot_free();
  if (ep.out_f32) {
    uint8_t* o = slot + lane * 128;
    if (ep.residual) {  // staged f32 residual at the output positions
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 r = *reinterpret_cast<const float4*>(o + ((q ^ sw128) * 16));
        v[4 * q + 0] += r.x;
        v[4 * q + 1] += r.y;
        v[4 * q + 2] += r.z;
        v[4 * q + 3] += r.w;
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<float4*>(o + ((q ^ sw128) * 16)) =
          make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
    uint8_t* o = slot + lane * 64;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
      w.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
      w.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
      w.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
      *reinterpret_cast<uint4*>(o + ((q ^ sw64) * 16)) = w;
    }
  }
  fence_proxy_async_shared();
  __syncwarp();
  if (lane == 0) {
    if (ep.flags & kEpiAccumulate)
      tma_reduce_add_2d(tmOut, slot, col0, row0);
    else
      tma_store_2d(tmOut, slot, col0, row0);
    if (aux_out) tma_store_2d(tmAux, slot + 2048, col0, row0);
    bulk_commit_group();
  }
}

template <int BN, bool A_MN, bool B_MN, int kSlots, bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tcgen05(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmOut,
                      const __grid_constant__ CUtensorMap tmAux,
                      const __grid_constant__ CUtensorMap tmIn, GemmEpilogue ep, int M, int N,
                      int K, int k_splits, int use_tma_store, int in_kind, uint32_t* err) {
  using Cfg = GemmCfg<BN, kSlots, kPair>;
  constexpr int S = Cfg::kStages;
  // Work units: single CTAs over 128 x BN tiles, or CTA pairs over 256 x BN
  // tiles (this CTA's rows start at crank * 128 within the tile).
  constexpr int kTM = kPair ? 2 * kBM : kBM;
  const uint32_t crank = kPair ? cluster_ctarank() : 0u;
  const int unit = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128B-swizzled tiles need 1024-byte alignment.
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + S * Cfg::kStageBytes;
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(staging + Cfg::kStagingBytes);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  const int tiles_m = (M + kTM - 1) / kTM;
  const int tiles_n = (N + BN - 1) / BN;
  const int k_blocks_total = (K + kBK - 1) / kBK;
  const int kb_per_split = (k_blocks_total + k_splits - 1) / k_splits;
  const int num_tiles = tiles_m * tiles_n * k_splits;
  const uint64_t limit = g_wait_limit_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->tmem_full[a], 1);
      // pair: the even CTA's barrier collects the epilogue warps of both CTAs
      mbar_init(&ctl->tmem_empty[a], kPair ? 2 * kEpiWarps : kEpiWarps);
    }
    mbar_init(&ctl->drain, 1);
    for (int i = 0; i < kEpiWarps * 2; ++i) mbar_init(&ctl->epi_in[i], 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (use_tma_store) {
      tma_prefetch_desc(&tmOut);
      tma_prefetch_desc(&tmAux);
      if (in_kind != kInNone) tma_prefetch_desc(&tmIn);
    }
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair<Cfg::kTmemCols>(&ctl->tmem_base);
      tmem_relinquish_pair();
    } else {
      tmem_alloc<Cfg::kTmemCols>(&ctl->tmem_base);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // pair: both CTAs' barriers are initialised before either signals the other
  if constexpr (kPair) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  // the prologue above may overlap the previous kernel of the stream; global
  // memory is touched only from here on
  pdl_wait();
  pdl_trigger();
  volatile uint32_t* abort_flag = &ctl->abort;

  auto tile_coords = [&](int t, int& tm, int& tn, int& ks) {
    ks = t % k_splits;
    int mn = t / k_splits;
    tn = mn % tiles_n;
    tm = mn / tiles_n;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = unit; t < num_tiles && ok; t += units) {
        int tm, tn, ks;
        tile_coords(t, tm, tn, ks);
        const int kb0 = ks * kb_per_split;
        const int kb1 = min(k_blocks_total, kb0 + kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait_bounded(&ctl->empty[s], ph ^ 1, abort_flag, err, limit)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + s * Cfg::kStageBytes;
          uint8_t* b_dst = a_dst + Cfg::kATileBytes;
          const int k0 = kb * kBK;
          if constexpr (kPair) {
            // both CTAs' bytes complete on the even CTA's barrier; only the
            // even CTA arrives (with the pair's byte count)
            if (crank == 0) mbar_arrive_expect_tx(&ctl->full[s], 2 * Cfg::kStageBytes);
            const int m0 = tm * kTM + (int)crank * kBM;
            const int n0 = tn * BN + (int)crank * (BN / 2);
            if (A_MN) {
              tma_load_2d_pair(a_dst, &tmA, &ctl->full[s], m0, k0);
              tma_load_2d_pair(a_dst + 64 * 128, &tmA, &ctl->full[s], m0 + 64, k0);
            } else {
              tma_load_2d_pair(a_dst, &tmA, &ctl->full[s], k0, m0);
            }
            if (B_MN) {
#pragma unroll
              for (int c = 0; c < BN / 128; ++c)
                tma_load_2d_pair(b_dst + c * 64 * 128, &tmB, &ctl->full[s], n0 + c * 64, k0);
            } else {
              tma_load_2d_pair(b_dst, &tmB, &ctl->full[s], k0, n0);
            }
            continue;
          }
          mbar_arrive_expect_tx(&ctl->full[s], Cfg::kStageBytes);
          if (A_MN) {
            tma_load_2d(a_dst, &tmA, &ctl->full[s], tm * kBM, k0);
            tma_load_2d(a_dst + 64 * 128, &tmA, &ctl->full[s], tm * kBM + 64, k0);
          } else {
            tma_load_2d(a_dst, &tmA, &ctl->full[s], k0, tm * kBM);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(b_dst + c * 64 * 128, &tmB, &ctl->full[s], tn * BN + c * 64, k0);
          } else {
            tma_load_2d(b_dst, &tmB, &ctl->full[s], k0, tn * BN);
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) for copies already in flight before leaving.
        for (int s = 0; s < S; ++s) {
          uint64_t t0 = global_timer_ns();
          while (!mbar_try_wait(&ctl->full[s], ((it - 1 - s) / S) & 1)) {
            if (global_timer_ns() - t0 > 100000000ull) break;
          }
        }
      }
    }
    __syncwarp();  // reconverge the warp before the CTA-wide barrier below
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // pair: the even CTA issues the pair's MMAs; the odd CTA's MMA warp idles
    if ((!kPair || crank == 0) && elect_one_sync()) {
      constexpr uint32_t idesc = make_idesc_bf16(kTM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      uint32_t it = 0;
      uint32_t local_tile = 0;
      bool ok = true;
      bool issued = false;
      for (int t = unit; t < num_tiles && ok; t += units, ++local_tile) {
        int tm, tn, ks;
        tile_coords(t, tm, tn, ks);
        const int kb0 = ks * kb_per_split;
        const int kb1 = min(k_blocks_total, kb0 + kb_per_split);
        const uint32_t acc = local_tile & 1;
        const uint32_t acc_ph = (local_tile >> 1) & 1;
        if (!mbar_wait_bounded(&ctl->tmem_empty[acc], acc_ph ^ 1, abort_flag, err, limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait_bounded(&ctl->full[s], ph, abort_flag, err, limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t b_addr = a_addr + Cfg::kATileBytes;
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            uint64_t adesc, bdesc;
            if (A_MN)
              adesc = make_sdesc_sw128(a_addr + j * 2048, 64 * 128, 1024);
            else
              adesc = make_sdesc_sw128(a_addr + j * 32, 16, 1024);
            if (B_MN)
              bdesc = make_sdesc_sw128(b_addr + j * 2048, 64 * 128, 1024);
            else
              bdesc = make_sdesc_sw128(b_addr + j * 32, 16, 1024);
            if constexpr (kPair)
              umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb > kb0 || j > 0) ? 1u : 0u);
            else
              umma_bf16(d_tmem, adesc, bdesc, idesc, (kb > kb0 || j > 0) ? 1u : 0u);
            issued = true;
          }
          // smem stage free once these MMAs finish (pair: in both CTAs)
          if constexpr (kPair)
            umma_commit_pair(&ctl->empty[s], 0x3);
          else
            umma_commit(&ctl->empty[s]);
        }
        if (!ok) break;
        // accumulator ready for the epilogue (pair: both CTAs' halves)
        if constexpr (kPair)
          umma_commit_pair(&ctl->tmem_full[acc], 0x3);
        else
          umma_commit(&ctl->tmem_full[acc]);
      }
      if (!ok && issued) {
        if constexpr (kPair)
          umma_commit_pair(&ctl->drain, 0x1);
        else
          umma_commit(&ctl->drain);
        uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&ctl->drain, 0)) {
          if (global_timer_ns() - t0 > 100000000ull) break;
        }
      }
    }
    __syncwarp();  // reconverge the warp before the CTA-wide barrier below
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int ew = warp - 2;              // epilogue warp 0..7
    const int half = ew / 4;              // which half of the tile's columns
    constexpr int kChunks = BN / 32 / 2;  // 32-column chunks per warp and tile
    uint8_t* stage = staging + ew * kSlots * kSlotBytes;
    uint64_t* in_bar = &ctl->epi_in[ew * 2];
    const float alpha = ep.alpha_ptr ? ep.alpha * __ldg(ep.alpha_ptr) : ep.alpha;
    const bool tma_in = use_tma_store && in_kind != kInNone;
    const int my_tiles = unit < num_tiles ? (num_tiles - 1 - unit) / units + 1 : 0;
    const int total = my_tiles * kChunks;
    // chunk j of this warp: tile unit + (j / kChunks) * units, column chunk j % kChunks
    auto chunk_at = [&](int j, int& row0, int& col0) -> bool {
      int tm, tn, ks;
      tile_coords(unit + (j / kChunks) * units, tm, tn, ks);
      row0 = tm * kTM + (int)crank * kBM + q * 32;
      col0 = tn * BN + (half * kChunks + j % kChunks) * 32;
      return col0 < N && row0 < M && ks * kb_per_split < k_blocks_total;
    };
    // TMA prefetch of chunk j's epilogue input into its slot (lane 0 issues)
    auto issue_in = [&](int j) -> bool {
      int row0, col0;
      if (!chunk_at(j, row0, col0)) return false;
      if (lane == 0) {
        uint64_t* bar = &in_bar[j & 1];
        uint8_t* slot = stage + (j & 1) * kSlotBytes;
        if (in_kind == kInResidual) {
          mbar_arrive_expect_tx(bar, 4096);
          tma_load_2d(slot, &tmIn, bar, col0, row0);
        } else {
          mbar_arrive_expect_tx(bar, 2048);
          tma_load_2d(slot + 2048, &tmIn, bar, col0, row0);
        }
      }
      return true;
    };
    // one N tile: every chunk cc of this warp has the same columns, so its
    // column sums accumulate in registers and leave with one atomic per CTA
    const bool keep_sums = (ep.colsum || ep.colsumsq) && tiles_n == 1 && k_splits == 1;
    float cs_acc[kChunks], cq_acc[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) cs_acc[c] = cq_acc[c] = 0.f;
    bool prev_stored = false;  // chunk j-1 committed a store group (its slot may be in flight)
    uint32_t in_ph = 0;    // parity of the next completion of each slot's barrier
    uint32_t pending = 0;  // slots with an input load issued but not yet consumed
    if (tma_in && total > 0 && issue_in(0)) pending |= 1u;
    bool aborted = false;
    for (int j = 0; j < total; ++j) {
      const int cc = j % kChunks;
      const uint32_t local_tile = (uint32_t)(j / kChunks);
      const uint32_t acc = local_tile & 1;
      if (cc == 0) {
        const bool ok =
            mbar_wait_bounded(&ctl->tmem_full[acc], (local_tile >> 1) & 1, abort_flag, err, limit);
        if (!__all_sync(0xffffffffu, ok)) {  // keep the warp converged for tcgen05.ld
          aborted = true;
          break;
        }
        tc_fence_after();
      }
      int row0, col0;
      const bool live = chunk_at(j, row0, col0);
      uint32_t r[32];
      tmem_ld_32cols(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN +
                         (uint32_t)((half * kChunks + cc) * 32),
                     r);
      tmem_ld_wait();
      if (cc == kChunks - 1) {
        // Last read of this accumulator by this warp: hand it back early
        // (pair: to the even CTA, whose MMA warp reuses both halves).
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (kPair)
            mbar_arrive_cluster(&ctl->tmem_empty[acc], 0);
          else
            mbar_arrive(&ctl->tmem_empty[acc]);
        }
      }
      if (use_tma_store) {
        // Slot j&1 was last read by the store of chunk j-2. With epilogue
        // inputs, the other slot (last read by chunk j-1's store) is about to
        // receive chunk j+1's input, so every store must have read its slot.
        // Without inputs only chunk j-2's store must have: chunk j-1's store
        // (the newest group) may still be reading while chunk j is computed.
        if (kSlots == 2) {
          if (lane == 0) {
            if (tma_in || !prev_stored)
              bulk_wait_group_read<0>();
            else
              bulk_wait_group_read<1>();
          }
          __syncwarp();
        }
        if (tma_in && j + 1 < total && issue_in(j + 1)) pending |= 1u << ((j + 1) & 1);
      }
      prev_stored = live && use_tma_store;
      if (!live) continue;
      if (use_tma_store) {
        uint8_t* slot = stage + (kSlots == 2 ? (j & 1) : 0) * kSlotBytes;
        if (tma_in) {
          const uint32_t sb = (uint32_t)(j & 1);
          const bool ok = mbar_wait_bounded(&in_bar[sb], (in_ph >> sb) & 1u, abort_flag, err, limit);
          in_ph ^= 1u << sb;
          pending &= ~(1u << sb);
          if (!__all_sync(0xffffffffu, ok)) {
            aborted = true;
            break;
          }
        }
        float* csk = nullptr;
        float* cqk = nullptr;
        if (keep_sums) {
#pragma unroll
          for (int c = 0; c < kChunks; ++c)
            if (c == cc) {
              csk = &cs_acc[c];
              cqk = &cq_acc[c];
            }
        }
        epilogue_chunk_tma(ep, alpha, &tmOut, &tmAux, slot, row0, col0, lane, N, r, kSlots == 1,
                           csk, cqk);
      } else {
        epilogue_chunk(ep, row0 + lane, col0, M, N, r);
      }
    }
    if (aborted && lane == 0) {
      // give input loads still in flight a bounded chance to land before exit
      for (uint32_t sb = 0; sb < 2; ++sb) {
        if (!(pending & (1u << sb))) continue;
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&in_bar[sb], (in_ph >> sb) & 1u)) {
          if (global_timer_ns() - t0 > 100000000ull) break;
        }
      }
    }
    if (keep_sums && !aborted) {
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        const int col = (half * kChunks + c) * 32 + lane;
        if (col < N) {
          if (ep.colsum) atomicAdd(ep.colsum + col, cs_acc[c]);
          if (ep.colsumsq) atomicAdd(ep.colsumsq + col, cq_acc[c]);
        }
      }
    }
    if (use_tma_store && lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  // pair: neither CTA leaves (freeing the shared memory and TMEM the other's
  // MMAs and barriers address) before both are done
  if constexpr (kPair) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair)
      tmem_dealloc_pair<Cfg::kTmemCols>(tmem_base);
    else
      tmem_dealloc<Cfg::kTmemCols>(tmem_base);
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

EncodeTiledFn get_encode_fn() {
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

}  // namespace

// 2D bf16 tensor map: inner dimension `inner` (contiguous), `outer` rows with
// row pitch `ld` elements; box = box_inner x box_outer, 128-byte swizzle.
static thread_local char g_tmap_fail[192];
const char* tmap_failure_detail() { return g_tmap_fail; }

bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t ld, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    snprintf(g_tmap_fail, sizeof(g_tmap_fail), "cuTensorMapEncodeTiled unavailable");
    return false;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    snprintf(g_tmap_fail, sizeof(g_tmap_fail),
             "CUresult %d base=%p inner=%llu outer=%llu ld=%llu box=%ux%u", (int)r, base,
             (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)ld,
             box_inner, box_outer);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  });
  return n;
}

static std::atomic<uint64_t> g_launches{0};
void note_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }
uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }
void reset_launch_count() { g_launches.store(0); }

static uint32_t* g_err_host = nullptr;
static uint32_t* g_err_dev = nullptr;
uint32_t* default_err_word() {
  static std::once_flag once;
  std::call_once(once, [] {
    void* hp = nullptr;
    if (cudaHostAlloc(&hp, 64, cudaHostAllocMapped) == cudaSuccess) {
      g_err_host = static_cast<uint32_t*>(hp);
      *g_err_host = 0;
      void* dp = nullptr;
      if (cudaHostGetDevicePointer(&dp, hp, 0) == cudaSuccess) g_err_dev = static_cast<uint32_t*>(dp);
    }
  });
  return g_err_dev;
}
uint32_t read_kernel_error() {
  default_err_word();
  return g_err_host ? *reinterpret_cast<volatile uint32_t*>(g_err_host) : 0u;
}
void clear_kernel_error() {
  default_err_word();
  if (g_err_host) *reinterpret_cast<volatile uint32_t*>(g_err_host) = 0u;
}

void set_wait_limit_ns(uint64_t ns) {
  cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns));
}

// Output-chunk tensor map: box 32 x 32, 128B swizzle for f32 rows of 128 B,
// 64B swizzle for bf16 rows of 64 B.
static bool make_out_tmap(CUtensorMap* map, void* base, bool f32, uint64_t cols, uint64_t rows,
                          uint64_t ld) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const uint64_t es = f32 ? 4 : 2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * es};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base,
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static thread_local const char* g_gemm_fail = nullptr;
const char* gemm_failure_detail() { return g_gemm_fail ? g_gemm_fail : ""; }

// One dynamic shared-memory opt-in per kernel instance and device (the
// template parameters key the static: every instance has the same type).
template <int BN, bool A_MN, bool B_MN, int kSlots, bool kPair>
static cudaError_t smem_opt_in() {
  auto kern = gemm_bf16_tcgen05<BN, A_MN, B_MN, kSlots, kPair>;
  const int bytes = GemmCfg<BN, kSlots, kPair>::kSmemBytes;
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_relaxed) & bit) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit);
  return e;
}

// Launch one kernel instance: plain grid, or (pair) a grid of (2,1,1) clusters.
template <int BN, bool A_MN, bool B_MN, int kSlots, bool kPair>
static cudaError_t launch_instance(const GemmArgs& g, cudaStream_t stream, const CUtensorMap& tmA,
                                   const CUtensorMap& tmB, const CUtensorMap& tmOut,
                                   const CUtensorMap& tmAux, const CUtensorMap& tmIn, int use_tma,
                                   int in_kind, uint32_t* err) {
  auto kern = gemm_bf16_tcgen05<BN, A_MN, B_MN, kSlots, kPair>;
  constexpr int smem = GemmCfg<BN, kSlots, kPair>::kSmemBytes;
  cudaError_t e = smem_opt_in<BN, A_MN, B_MN, kSlots, kPair>();
  if (e != cudaSuccess) return e;
  constexpr int tm = kPair ? 2 * kBM : kBM;
  const int tiles = ((g.M + tm - 1) / tm) * ((g.N + BN - 1) / BN) * g.k_splits;
  if constexpr (kPair) {
    const int pairs = std::min(tiles, num_sms() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmOut, tmAux, tmIn, g.ep, g.M, g.N, g.K,
                              g.k_splits, use_tma, in_kind, err);
  } else {
    const int grid = tiles < num_sms() ? tiles : num_sms();
    return launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, tmA, tmB, tmOut, tmAux,
                      tmIn, g.ep, g.M, g.N, g.K, g.k_splits, use_tma, in_kind, err);
  }
}

// FLODL_GEMM_EPI_SLOTS: 0 (unset) = automatic, 1 or 2 = staging slots per
// epilogue warp for epilogues without an input (read once per process).
static int epi_slots_override() {
  static const int v = [] {
    const char* e = std::getenv("FLODL_GEMM_EPI_SLOTS");
    const int k = e ? std::atoi(e) : 0;
    return (k == 1 || k == 2) ? k : 0;
  }();
  return v;
}

template <int BN, bool A_MN, bool B_MN, bool kPair = false>
static cudaError_t launch_gemm_t(const GemmArgs& g, cudaStream_t stream) {
  CUtensorMap tmA, tmB;
  // A tile: 128 (M) x 64 (K)
  bool ok;
  if (A_MN)
    ok = make_tmap_bf16_2d(&tmA, g.A, g.M, g.K, g.lda, 64, kBK);
  else
    ok = make_tmap_bf16_2d(&tmA, g.A, g.K, g.M, g.lda, kBK, kBM);
  if (!ok) {
    g_gemm_fail = tmap_failure_detail();
    return cudaErrorInvalidValue;
  }
  if (B_MN)
    ok = make_tmap_bf16_2d(&tmB, g.B, g.N, g.K, g.ldb, 64, kBK);
  else
    ok = make_tmap_bf16_2d(&tmB, g.B, g.K, g.N, g.ldb, kBK, kPair ? BN / 2 : BN);
  if (!ok) {
    g_gemm_fail = tmap_failure_detail();
    return cudaErrorInvalidValue;
  }

  // TMA-store epilogue when every tensor it moves is 16-byte aligned (base and
  // row pitch) and the combination fits a 4 KB staging slot: f32 out (+ f32
  // residual in), or bf16 out (+ bf16 GELU' out for GELU, or bf16
  // GELU' operand in). Anything else takes the direct-store epilogue.
  CUtensorMap tmOut, tmAux, tmIn;
  std::memset(&tmOut, 0, sizeof(tmOut));
  std::memset(&tmAux, 0, sizeof(tmAux));
  std::memset(&tmIn, 0, sizeof(tmIn));
  auto aligned = [](const void* p, int ld, int es) {
    return (reinterpret_cast<uintptr_t>(p) % 16 == 0) && ((uint64_t)ld * es) % 16 == 0;
  };
  const bool f32 = g.ep.out_f32 != 0;
  const bool aux_out = (g.ep.flags & kEpiGelu) && g.ep.aux;
  const bool dgelu = (g.ep.flags & kEpiDGelu) != 0;
  const bool res = g.ep.residual != nullptr;
  bool use_tma = aligned(g.ep.out, g.ep.ld_out, f32 ? 4 : 2);
  if (aux_out || dgelu) use_tma = use_tma && !f32 && aligned(g.ep.aux, g.ep.ld_aux, 2);
  if (res) use_tma = use_tma && f32 && aligned(g.ep.residual, g.ep.ld_res, 4);
  if (aux_out && dgelu) use_tma = false;
  int in_kind = kInNone;
  if (use_tma) use_tma = make_out_tmap(&tmOut, g.ep.out, f32, g.N, g.M, g.ep.ld_out);
  if (use_tma && aux_out) use_tma = make_out_tmap(&tmAux, g.ep.aux, false, g.N, g.M, g.ep.ld_aux);
  if (use_tma && res) {
    use_tma = make_out_tmap(&tmIn, const_cast<float*>(g.ep.residual), true, g.N, g.M, g.ep.ld_res);
    in_kind = kInResidual;
  } else if (use_tma && dgelu) {
    use_tma = make_out_tmap(&tmIn, g.ep.aux, false, g.N, g.M, g.ep.ld_aux);
    in_kind = kInAux;
  }
  if (!use_tma) in_kind = kInNone;
  if ((g.ep.colsum || g.ep.colsumsq) && !use_tma) {
    g_gemm_fail = "fused column sums need the TMA-store epilogue (aligned output/aux)";
    return cudaErrorInvalidValue;
  }
  uint32_t* err = g.err ? g.err : default_err_word();
  // Epilogues without an input take a single staging slot (the previous
  // chunk's store reads it while this chunk is computed) and one more operand
  // stage where that fits; two slots measured slower (qkv 28.5 -> 30.1 us,
  // fc1 58.8 -> 62.6 us). FLODL_GEMM_EPI_SLOTS=2 selects two slots.
  const bool two = in_kind != kInNone || epi_slots_override() == 2;
  cudaError_t e =
      !two ? launch_instance<BN, A_MN, B_MN, 1, kPair>(g, stream, tmA, tmB, tmOut, tmAux, tmIn,
                                                       use_tma ? 1 : 0, in_kind, err)
           : launch_instance<BN, A_MN, B_MN, 2, kPair>(g, stream, tmA, tmB, tmOut, tmAux, tmIn,
                                                       use_tma ? 1 : 0, in_kind, err);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLODL_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// FLODL_GEMM_PAIR=0 turns the CTA-pair tiles off (read once per process).
static bool pair_tiles_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLODL_GEMM_PAIR");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Shortest reduction per tile that takes CTA-pair tiles (FLODL_GEMM_PAIR_MIN_K).
static int pair_min_k() {
  static const int k = [] {
    const char* v = std::getenv("FLODL_GEMM_PAIR_MIN_K");
    return v ? std::max(64, std::atoi(v)) : 1024;
  }();
  return k;
}

cudaError_t launch_gemm(const GemmArgs& g, cudaStream_t stream) {
  g_gemm_fail = nullptr;
  if (g.M <= 0 || g.N <= 0 || g.K <= 0 || g.k_splits < 1) {
    g_gemm_fail = "empty problem or bad split";
    return cudaErrorInvalidValue;
  }
  const bool wide = g.N >= 256 && g.bn != 128;
  // 192-column tiles when they leave fewer idle SM-slots in the last wave:
  // estimated time ~ waves(tiles) * tile width (e.g. N = 1536 at M = 16384:
  // 6 waves of 256 vs 7 waves of 192, 7/8 of the time)
  bool w192 = false;
  if (wide && g.bn == 0 && g.k_splits == 1) {
    const int tm = (g.M + kBM - 1) / kBM, sms = num_sms();
    const long t256 = (long)tm * ((g.N + 255) / 256), t192 = (long)tm * ((g.N + 191) / 192);
    w192 = ((t192 + sms - 1) / sms) * 192 < ((t256 + sms - 1) / sms) * 256;
  }
  // CTA pairs (256-row tiles, half the operand bytes per CTA and K step) for
  // wide problems with enough rows and a long reduction per tile: with
  // K >= 1024 the main loop is bound by operand bytes per SM, which the pair
  // halves; shorter loops (K = 512) measured faster on single-CTA tiles,
  // where fill latency and the epilogue dominate. bn = 128 / 256 force the
  // single-CTA tiles.
  const bool pair = wide && g.bn == 0 && g.M >= 512 && g.K / g.k_splits >= pair_min_k() &&
                    pair_tiles_enabled();
#define FL_GEMM_CASE(AMN, BMN)                                                   \
  if (g.a_mn == AMN && g.b_mn == BMN)                                           \
    return pair ? launch_gemm_t<256, AMN, BMN, true>(g, stream)                \
                : w192 ? launch_gemm_t<192, AMN, BMN>(g, stream)               \
                       : wide ? launch_gemm_t<256, AMN, BMN>(g, stream)        \
                              : launch_gemm_t<128, AMN, BMN>(g, stream);
  FL_GEMM_CASE(false, false)
  FL_GEMM_CASE(false, true)
  FL_GEMM_CASE(true, false)
  FL_GEMM_CASE(true, true)
#undef FL_GEMM_CASE
  return cudaErrorInvalidValue;
}

}  // namespace flodl
