// Thin inline-PTX layer for the Blackwell (sm_100a) execution model used by
// every hand-written kernel in this package: mbarriers with bounded waits,
// TMA tile loads (never with cluster multicast), tcgen05 MMA issue/commit,
// TMEM allocation and TMEM -> register loads.
//
// Every wait in this file is bounded by %globaltimer. A wait that runs out
// records an error code in a device word the host can read and returns false;
// callers then unwind (free TMEM, return) instead of hanging the GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <utility>

namespace flodl {

// ---------------------------------------------------------------- basics
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n"
      ".reg .b32 rx;\n"
      ".reg .pred px;\n"
      "elect.sync rx|px, %1;\n"
      "selp.b32 %0, 1, 0, px;\n"
      "}\n"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred;
}

// Error words. Kernels write a nonzero code here (first writer wins) when a
// bounded wait expires; the host polls it after synchronising.
enum KernelError : uint32_t {
  kErrNone = 0,
  kErrMbarTimeout = 1,
  kErrPeerTimeout = 2,
  kErrBadArgs = 3,
  kErrBadLabel = 4,  // a class target outside [0, V) that is not ignore_index
};

__device__ __forceinline__ void report_error(uint32_t* err, uint32_t code) {
  if (err) atomicCAS(err, 0u, code);
}

// ---------------------------------------------------------------- division by a launch constant
// Unsigned division of dividends below 2^31 by a divisor d (1 <= d <= 2^31)
// fixed at launch, as one multiply-high, one add and one shift: with
// s = ceil(log2 d) and m = floor(2^32 (2^s - d) / d) + 1, q = (umulhi(n, m) + n)
// >> s (Granlund and Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, section 4; n < 2^31 keeps the add from
// wrapping). Elementwise kernels that split a flat index into coordinates
// spend most of their issue slots on divisions otherwise.
struct FastDiv {
  uint32_t d = 1, m = 1, s = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t div) : d(div) {
    while ((1ull << s) < div) ++s;
    m = (uint32_t)((((1ull << s) - div) << 32) / div + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> s; }
};
constexpr int64_t kMaxFlatIndex = (int64_t)1 << 31;  // flat indices of FastDiv kernels

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels launched with launch_pdl may start (their prologue: barrier init,
// TMEM allocation, descriptor prefetch) while the previous kernel of the
// stream is still finishing; pdl_wait() blocks until that kernel completed and
// its memory is visible, so it comes before the first global access.
// pdl_trigger() lets the next PDL launch of the stream be scheduled once every
// CTA of this grid has started. Both are no-ops for an ordinary launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// FLODL_PDL=0 turns programmatic dependent launches off (read once per process).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete. Gives up after `limit_ns`
// nanoseconds, or immediately once *abort is set by another role of the same
// CTA, and returns false in both cases.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile uint32_t* abort, uint32_t* err,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (((++spins) & 63u) == 0u) {
      if (abort && *abort) return false;
      if (global_timer_ns() - t0 > limit_ns) {
        if (abort) *abort = 1u;
        report_error(err, kErrMbarTimeout);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA
// 2D tile load global -> shared, completion counted on `bar` (complete_tx).
// The innermost coordinate x must be a multiple of 16 bytes / element size.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3D tile load (used for batched operands: x inner, y rows, z batch).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 2D tile store shared -> global (bulk-group completion). Out-of-range rows and
// columns of the box are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src,
                                             int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}

// 2D tile reduce-add shared -> global (f32 accumulation, e.g. split-K).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src,
                                                  int32_t x, int32_t y) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N committed bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed bulk groups are still in flight.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
template <uint32_t kCols>
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result) {
  static_assert(kCols >= 32 && (kCols & (kCols - 1)) == 0 && kCols <= 512, "TMEM columns");
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(kCols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

template <uint32_t kCols>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(kCols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (bf16/f16 inputs, f32 accumulate).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc): A operand read from tensor memory.
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- CTA pairs
// Two CTAs of a (2,1,1) cluster share one tcgen05.mma (cta_group::2): the
// even CTA issues it, each CTA holds half of A (M rows) and half of B (N rows)
// at the same shared-memory offsets, and each CTA's TMEM holds its M half of
// the accumulator.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Arrive on the barrier at the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
  asm volatile(
      "{\n"
      ".reg .b32 ra;\n"
      "mapa.shared::cluster.u32 ra, %0, %1;\n"
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n"
      "}\n" ::"r"(smem_u32(bar)),
      "r"(rank)
      : "memory");
}
// TMA 2D load into this CTA's shared memory whose completed bytes are counted
// on the even CTA's barrier at `bar`'s offset (no multicast). The barrier's
// shared::cluster address in CTA 0 comes from mapa.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "{\n"
      ".reg .b32 rb;\n"
      "mapa.shared::cluster.u32 rb, %2, 0;\n"
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [rb];\n"
      "}\n" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
template <uint32_t kCols>
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result) {
  static_assert(kCols >= 32 && (kCols & (kCols - 1)) == 0 && kCols <= 512, "TMEM columns");
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(kCols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
template <uint32_t kCols>
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(kCols)
               : "memory");
}
// D (both CTAs' TMEM, M = 256) (+)= A * B with A/B halves in both CTAs.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at `bar`'s offset in every CTA of `cta_mask` once the
// pair MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Instruction descriptor, kind::f16 with bf16 A/B and f32 accumulator.
// a_mn / b_mn select MN-major (transposed) operands.
__host__ __device__ constexpr uint32_t make_idesc_bf16(uint32_t M, uint32_t N, uint32_t a_mn,
                                                       uint32_t b_mn) {
  return (1u << 4)            // D format: f32
         | (1u << 7)          // A format: bf16
         | (1u << 10)         // B format: bf16
         | (a_mn << 15)       // A major
         | (b_mn << 16)       // B major
         | ((N >> 3) << 17)   // N / 8
         | ((M >> 4) << 24);  // M / 16
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version bits.
// lbo/sbo in bytes.
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t smem_addr, uint32_t lbo,
                                                     uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for tcgen05
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// TMEM -> registers: 32 lanes x 32-bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// TMEM -> registers: 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_16cols(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// registers -> TMEM: 32 lanes x 32-bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_st_16cols(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Named barrier among a subset of warps (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- math helpers
// erf for the GEMM epilogues: Abramowitz & Stegun, Handbook of Mathematical
// Functions, eq. 7.1.28 (after Hastings):
//   erf(x) = 1 - 1 / (1 + a1 x + a2 x^2 + ... + a6 x^6)^16,  x >= 0,
//   |error| <= 3e-7,
// extended to x < 0 by oddness. One reciprocal and eleven multiply-adds; the
// outputs it feeds are rounded to bf16 (relative step 2^-8), far coarser than
// the approximation error. The polynomial is evaluated at min(|x|, 8), where
// the result is already 1 to single precision. The reciprocal is the hardware
// approximation (rel. error ~2^-23), negligible after the subtraction from 1.
__device__ __forceinline__ float erf_as7128(float x) {
  const float ax = fminf(fabsf(x), 8.0f);
  float p = 0.0000430638f;
  p = fmaf(p, ax, 0.0002765672f);
  p = fmaf(p, ax, 0.0001520143f);
  p = fmaf(p, ax, 0.0092705272f);
  p = fmaf(p, ax, 0.0422820123f);
  p = fmaf(p, ax, 0.0705230784f);
  p = fmaf(p, ax, 1.0f);
  p = p * p;  // ^2
  p = p * p;  // ^4
  p = p * p;  // ^8
  p = p * p;  // ^16
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(p));
  return copysignf(1.0f - r, x);
}

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erf_as7128(x * 0.70710678118654752f));
}
// GELU and its derivative together (the forward epilogue keeps GELU'(x) for
// the backward): g = x Phi(x), dg = Phi(x) + x phi(x), phi the normal density.
__device__ __forceinline__ void gelu_and_grad(float x, float& g, float& dg) {
  const float cdf = 0.5f * (1.0f + erf_as7128(x * 0.70710678118654752f));
  g = x * cdf;
  dg = cdf + x * (0.39894228040143268f * __expf(-0.5f * x * x));
}
// d/dx of the erf GELU.
__device__ __forceinline__ float gelu_erf_grad(float x) {
  const float cdf = 0.5f * (1.0f + erf_as7128(x * 0.70710678118654752f));
  const float pdf = 0.39894228040143268f * __expf(-0.5f * x * x);
  return cdf + x * pdf;
}

// Column sums of a 32x32 chunk held one row per lane (v[c] = element (lane, c)):
// a butterfly reduce-scatter leaves the sum of column `lane` in lane `lane`
// after 31 shuffles (each stage halves the columns a lane keeps; lanes with
// the stage's bit set keep the upper half).
__device__ __forceinline__ float chunk_column_sum(const float (&v)[32], int lane) {
  float a[16];
  {
    const bool up = lane & 16;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float send = up ? v[k] : v[k + 16];
      const float keep = up ? v[k + 16] : v[k];
      a[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  float b[8];
  {
    const bool up = lane & 8;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float send = up ? a[k] : a[k + 8];
      const float keep = up ? a[k + 8] : a[k];
      b[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  float c[4];
  {
    const bool up = lane & 4;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float send = up ? b[k] : b[k + 4];
      const float keep = up ? b[k + 4] : b[k];
      c[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
  }
  float d[2];
  {
    const bool up = lane & 2;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float send = up ? c[k] : c[k + 2];
      const float keep = up ? c[k + 2] : c[k];
      d[k] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
  }
  const bool up = lane & 1;
  const float send = up ? d[0] : d[1];
  const float keep = up ? d[1] : d[0];
  return keep + __shfl_xor_sync(0xffffffffu, send, 1);
}

// ---------------------------------------------------------------- packed f32x2
// sm_100 executes add/mul/fma on a pair of f32 values held in one 64-bit
// register pair as one instruction (`.f32x2`, round-to-nearest like the scalar
// forms), halving the issue slots of elementwise epilogue math.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_splat(float a) { return f2_pack(a, a); }
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// GELU and GELU' of two values with packed math. erf after Abramowitz &
// Stegun 7.1.26 (|error| <= 1.5e-7), whose exponential is the Gaussian factor
// that GELU' needs anyway, so one ex2 serves both:
//   z = |x| / sqrt(2),  t = 1 / (1 + p z),  e = exp(-x^2 / 2)
//   erfc(z) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) e
//   Phi(x) = 1/2 + sign(x) (1/2 - erfc(z) / 2)
//   GELU(x) = x Phi(x),  GELU'(x) = Phi(x) + x e / sqrt(2 pi)
// The sign is copied with integer ops; the polynomial and products run as
// f32x2 pairs.
__device__ __forceinline__ void gelu_and_grad2(float x0, float x1, float& g0, float& g1,
                                               float& d0, float& d1) {
  constexpr float kP = 0.3275911f * 0.70710678118654752f;  // p / sqrt(2): t from |x|
  constexpr float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f,
                  a4 = -1.453152027f, a5 = 1.061405429f;
  const uint64_t x = f2_pack(x0, x1);
  const uint64_t den = f2_fma(f2_pack(fabsf(x0), fabsf(x1)), f2_splat(kP), f2_splat(1.0f));
  float n0, n1, t0, t1;
  f2_unpack(den, n0, n1);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t0) : "f"(n0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t1) : "f"(n1));
  const uint64_t t = f2_pack(t0, t1);
  uint64_t poly = f2_fma(f2_splat(a5), t, f2_splat(a4));
  poly = f2_fma(poly, t, f2_splat(a3));
  poly = f2_fma(poly, t, f2_splat(a2));
  poly = f2_fma(poly, t, f2_splat(a1));
  poly = f2_mul(poly, t);
  // exp(-x^2 / 2) = 2^(-x^2 log2(e) / 2)
  const uint64_t arg = f2_mul(x, f2_mul(x, f2_splat(-0.72134752044448170f)));
  float q0, q1, e0, e1;
  f2_unpack(arg, q0, q1);
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(q0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(q1));
  const uint64_t e = f2_pack(e0, e1);
  // h = 1/2 - erfc / 2 in [0, 1/2], then Phi = 1/2 + copysign(h, x)
  float h0, h1;
  f2_unpack(f2_fma(f2_mul(poly, e), f2_splat(-0.5f), f2_splat(0.5f)), h0, h1);
  const float s0 = __uint_as_float(__float_as_uint(h0) | (__float_as_uint(x0) & 0x80000000u));
  const float s1 = __uint_as_float(__float_as_uint(h1) | (__float_as_uint(x1) & 0x80000000u));
  const uint64_t cdf = f2_add(f2_pack(s0, s1), f2_splat(0.5f));
  f2_unpack(f2_mul(x, cdf), g0, g1);
  f2_unpack(f2_fma(f2_mul(x, e), f2_splat(0.39894228040143268f), cdf), d0, d1);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// bf16 -> f32 is exact: a bf16 is the upper half of the f32 of the same value,
// so two shifts/masks on the integer pipe unpack a pair.
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) {
  return __uint_as_float((uint32_t)__bfloat16_as_ushort(v) << 16);
}

// Vectorised fire-and-forget fp32 add into global memory (sm_90+).
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

}  // namespace flodl
