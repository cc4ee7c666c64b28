// Peer-memory communicator for one NVLink/NVSwitch node, and the fused
// collective kernels that run over it.
//
// Symmetric memory: every rank cudaMalloc's the same-sized regions (parameter
// arena, gradient arena, bf16 shadow arena, signal words) and exports CUDA IPC
// handles; each rank opens its peers' handles, so a kernel on rank r can load
// from / store to any rank's region over NVLink. NCCL (or the torch.distributed
// store) is only used to exchange the handles.
//
// Synchronisation: there is no grid-wide handshake. Block b of a launch meets
// block b of the same launch on every peer (all ranks launch the same grid):
// it publishes a per-(slot, block) phase counter into every peer's flag word
// with a system-scope release store (lane p stores to peer p, so the world
// stores go out in parallel) and waits until every peer's counter for that
// block reached the same phase (lane p polls the word peer p writes). A launch
// has a start meeting (inputs of every rank are ready) and an end meeting
// (every peer finished reading this rank's inputs and writing its results
// here). The element mapping of block b is identical on every rank, so what a
// block may overwrite after its end meeting is exactly what the peers' block b
// read. Every wait is bounded by %globaltimer (and gives up early once the
// communicator's error word is set); on expiry the kernel records an error
// code in host-mapped memory and returns.
//
// Sharding: a range of n float4 is cut into `world` shards of ceil(n/world);
// rank r owns shard r. Only rank r reads or writes the shard-r elements of any
// rank's gradient or parameter buffer during a two-shot launch, which is why
// a reduce-scatter can write its result straight back in place.
//
// Kernels:
//  ar_update (AdamW / SGD)   per DDP bucket, the reference's
//      "all_reduce_gradients (Avg) then optimizer.step()" (flodl/src/distributed/
//      ddp.rs:249-260 + nn/optim/adam.rs:183-245, sgd.rs) as ONE launch:
//      two-shot: reduce shard r from all peers (peer loads), update it, store
//      the f32 weights and bf16 shadow into every rank (peer stores);
//      one-shot (small buckets): every rank reduces the whole bucket in the
//      same peer order and updates it locally (bitwise-identical replicas).
//      After the end meeting each rank clears its gradient bucket.
//  reduce_scatter + clip_apply   the same with global-norm clipping
//      (flodl-sys/ops_training.cpp:948-985): buckets only average their shard
//      in place and add its sum of squares; the apply launch exchanges the
//      partial sums, derives the clip coefficient and updates every bucket.
//  weighted_average   cluster parameter averaging (worker/sync.rs:130-236):
//      params <- sum_i (m_i / sum m) W_i with m_i = n_i^gamma, f32 buffers
//      <- mover-weighted mean; the mass exchange rides the start meeting and
//      the divergence partials of every rank are computed in the same pass.
//  broadcast_pull     initial parameter broadcast (rank_entry.rs:619-623).
//  all_reduce         plain sum/avg all-reduce of a symmetric buffer.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>

#include "../kernels/sm100_ptx.cuh"
#include "peer_comm.h"

namespace flodl {

namespace {

constexpr int kIlp = 4;  // float4 elements per thread in flight per loop iteration

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_cg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ void add4(float4& a, const float4 b) {
  a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
}
__device__ __forceinline__ void scale4(float4& a, float s) {
  a.x *= s; a.y *= s; a.z *= s; a.w *= s;
}
__device__ __forceinline__ float dot4(const float4 a) {
  return a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
}
__device__ __forceinline__ uint2 bf16x4(const float4 v) {
  uint2 s;
  s.x = pack_bf16x2(v.x, v.y);
  s.y = pack_bf16x2(v.z, v.w);
  return s;
}

// Wait until *p >= target (wrap-safe). Gives up when the deadline passes or
// the communicator's error word is already set (another block timed out).
__device__ __forceinline__ bool wait_ge(const uint32_t* p, uint32_t target, uint64_t limit_ns,
                                        uint32_t* err) {
  uint64_t t0 = 0;
  uint32_t spins = 0;
  while ((int32_t)(ld_acquire_sys(p) - target) < 0) {
    if ((++spins & 255u) == 0u) {
      if (err && *reinterpret_cast<volatile uint32_t*>(err) != 0u) return false;
      if (t0 == 0) {
        t0 = global_timer_ns();
      } else if (global_timer_ns() - t0 > limit_ns) {
        if (err) atomicCAS_system(err, 0u, (uint32_t)kErrPeerTimeout);
        return false;
      }
    }
  }
  return true;
}

// Signal words (u32) of one rank's symmetric signal region:
//   flags[slot][block][src] : phase counter of (slot, block) on rank src (peer stores)
//   phase[slot][block]      : this rank's phase counter of (slot, block) (local)
//   mass[slot][src][2]      : f32 bits published by rank src (mass, mover / sumsq)
//   part[block][src][2]     : f32 divergence partials computed by rank src for this rank
//   count[slot]             : local: blocks that consumed the clip accumulator
struct SigLayout {
  static constexpr int kFlags = 0;
  static constexpr int kPhase = kFlags + kMaxSlots * kMaxBlocks * kMaxRanks;
  static constexpr int kMass = kPhase + kMaxSlots * kMaxBlocks;
  static constexpr int kPart = kMass + kMaxSlots * kMaxRanks * 2;
  static constexpr int kCount = kPart + kMaxBlocks * kMaxRanks * 2;
  static constexpr int kWords = kCount + kMaxSlots;
};

struct Handles {
  float* data[kMaxRanks];
  float* grad[kMaxRanks];
  __nv_bfloat16* shadow[kMaxRanks];
  uint32_t* sig[kMaxRanks];
};

__device__ __forceinline__ int flag_idx(int slot, int block, int src) {
  return SigLayout::kFlags + (slot * kMaxBlocks + block) * kMaxRanks + src;
}

// Meeting of block blockIdx.x with the same block of every peer on `slot`.
// Everything this block wrote before (locally or into peers) is visible to a
// peer block that passed the meeting, and vice versa. CTA-uniform result.
__device__ __forceinline__ bool meet(const Handles& h, int rank, int world, int slot,
                                  uint64_t limit, uint32_t* err) {
  __shared__ uint32_t ph_sh;
  uint32_t* sig = h.sig[rank];
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* c = sig + SigLayout::kPhase + slot * kMaxBlocks + blockIdx.x;
    const uint32_t ph = *c + 1u;
    *c = ph;
    ph_sh = ph;
  }
  __syncthreads();
  bool ok = true;
  if ((int)threadIdx.x < world) {
    const uint32_t ph = ph_sh;
    st_release_sys(h.sig[threadIdx.x] + flag_idx(slot, blockIdx.x, rank), ph);
    ok = wait_ge(sig + flag_idx(slot, blockIdx.x, threadIdx.x), ph, limit, err);
  }
  return __syncthreads_and(ok) != 0;
}

// Shard of `rank` in float4 units: [s0, s1); `per` = shard length.
struct Shard {
  int64_t b0, b1;  // whole range (float4)
  int64_t per;
  __device__ Shard(const FusedArgs& a) {
    b0 = a.start / 4;
    b1 = a.end / 4;
    per = (b1 - b0 + a.world - 1) / a.world;
  }
  __device__ int64_t s0(int r) const { return b0 + per * r; }
  __device__ int64_t s1(int r) const { return min(b1, b0 + per * (r + 1)); }
};

__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r += sh[i];
  __syncthreads();
  return r;
}

// ------------------------------------------------------------------ updates
// Per-element optimizer updates on a float4 of weights. `i` indexes the
// float4 in the arena (m/v/momentum buffers are arena-sized and local).
struct AdamWUpdate {
  float lr, b1, b2, eps, wd, bc1, bc2s;
  float* m;
  float* v;
  __device__ AdamWUpdate(const FusedArgs& a) {
    lr = *a.lr;
    const float t = *a.step;
    b1 = a.beta1;
    b2 = a.beta2;
    eps = a.eps;
    wd = a.wd;
    bc1 = 1.f - powf(a.beta1, t);
    bc2s = sqrtf(1.f - powf(a.beta2, t));
    m = a.m;
    v = a.v;
  }
  __device__ __forceinline__ void operator()(float4& p, const float4 g, int64_t i) const {
    float4 mv = reinterpret_cast<const float4*>(m)[i];
    float4 vv = reinterpret_cast<const float4*>(v)[i];
    float* pp = &p.x;
    const float* gg = &g.x;
    float* mm = &mv.x;
    float* vq = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      mm[k] = b1 * mm[k] + (1.f - b1) * gg[k];
      vq[k] = b2 * vq[k] + (1.f - b2) * gg[k] * gg[k];
      const float denom = sqrtf(vq[k]) / bc2s + eps;
      pp[k] = pp[k] * (1.f - lr * wd) - (lr / bc1) * mm[k] / denom;
    }
    reinterpret_cast<float4*>(m)[i] = mv;
    reinterpret_cast<float4*>(v)[i] = vv;
  }
};

struct SgdUpdate {
  float lr, wd, mom, damp;
  bool first, nesterov;
  float* buf;
  __device__ SgdUpdate(const FusedArgs& a) {
    lr = *a.lr;
    wd = a.wd;
    mom = a.momentum;
    damp = a.dampening;
    first = a.first ? (*a.first != 0.f) : false;
    nesterov = a.nesterov;
    buf = a.m;
  }
  __device__ __forceinline__ void operator()(float4& p, const float4 g, int64_t i) const {
    float4 bv = buf ? reinterpret_cast<const float4*>(buf)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    float* pp = &p.x;
    const float* gg = &g.x;
    float* bb = &bv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float d = gg[k] + wd * pp[k];
      if (buf) {
        bb[k] = first ? d : mom * bb[k] + (1.f - damp) * d;
        d = nesterov ? d + mom * bb[k] : bb[k];
      }
      pp[k] -= lr * d;
    }
    if (buf) reinterpret_cast<float4*>(buf)[i] = bv;
  }
};

__device__ __forceinline__ float grad_scale(const FusedArgs& a) {
  return (a.gscale ? *a.gscale : 1.f) / (float)a.world;
}

// Sum of the world gradients at the float4 indices idx[0..ILP) (fixed peer
// order 0..world-1, so every rank that sums the same element gets the same
// bits). W > 0: the world size is a compile-time constant and the loads of
// every peer are issued before the first add (W x ILP float4 in flight per
// thread); W == 0: any world size, one peer's loads in flight at a time.
template <int W, int ILP>
__device__ __forceinline__ void gather_sum(const Handles& h, int world, const int64_t* idx,
                                           const bool* live, float4* acc) {
  if constexpr (W > 0) {
    float4 x[W][ILP];
#pragma unroll
    for (int p = 0; p < W; ++p)
#pragma unroll
      for (int j = 0; j < ILP; ++j)
        x[p][j] = live[j] ? ld_cg4(h.grad[p] + 4 * idx[j]) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < ILP; ++j) {
      acc[j] = x[0][j];
#pragma unroll
      for (int p = 1; p < W; ++p) add4(acc[j], x[p][j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < ILP; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
    for (int p = 0; p < world; ++p) {
      float4 x[ILP];
#pragma unroll
      for (int j = 0; j < ILP; ++j)
        x[j] = live[j] ? ld_cg4(h.grad[p] + 4 * idx[j]) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < ILP; ++j) add4(acc[j], x[j]);
    }
  }
}

// float4 per thread and loop iteration for a compile-time world size (the
// gather keeps W x ILP float4 loads in flight).
template <int W>
struct IlpFor {
  static constexpr int value = W == 0 ? 4 : (W <= 2 ? 4 : (W <= 4 ? 2 : 1));
};

// Clear this rank's gradient elements that the peers' block blockIdx.x read:
// the block's positions in every shard (two-shot) or in the whole range.
__device__ __forceinline__ void clear_local_grads(const Handles& h, const FusedArgs& a,
                                                  const Shard& sh) {
  float4* gl = reinterpret_cast<float4*>(h.grad[a.rank]);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  if (a.oneshot) {
    for (int64_t i = sh.b0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < sh.b1; i += stride)
      gl[i] = z;
  } else {
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < sh.per; j += stride)
      for (int s = 0; s < a.world; ++s) {
        const int64_t i = sh.s0(s) + j;
        if (i < sh.s1(s)) gl[i] = z;
      }
  }
}

// ------------------------------------------------------------------ fused AR + update
template <class U, int W>
__global__ void __launch_bounds__(512, 2) ar_update_kernel(const __grid_constant__ FusedArgs a,
                                                 const __grid_constant__ Handles h) {
  constexpr int ILP = IlpFor<W>::value;
  if (!meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err)) return;
  const Shard sh(a);
  const int64_t lo = a.oneshot ? sh.b0 : sh.s0(a.rank);
  const int64_t hi = a.oneshot ? sh.b1 : sh.s1(a.rank);
  const U upd(a);
  const float gs = grad_scale(a);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < hi;
       i0 += ILP * stride) {
    int64_t idx[ILP];
    bool live[ILP];
#pragma unroll
    for (int j = 0; j < ILP; ++j) {
      idx[j] = i0 + j * stride;
      live[j] = idx[j] < hi;
    }
    float4 g[ILP];
    gather_sum<W, ILP>(h, a.world, idx, live, g);
#pragma unroll
    for (int j = 0; j < ILP; ++j) {
      if (!live[j]) break;
      const int64_t i = idx[j];
      float4 gj = g[j];
      scale4(gj, gs);
      float4 pv = reinterpret_cast<const float4*>(h.data[a.rank])[i];
      upd(pv, gj, i);
      const uint2 s = bf16x4(pv);
      if (a.oneshot) {
        reinterpret_cast<float4*>(h.data[a.rank])[i] = pv;
        if (h.shadow[a.rank]) reinterpret_cast<uint2*>(h.shadow[a.rank])[i] = s;
      } else {
        for (int p = 0; p < a.world; ++p) {
          const int q = (a.rank + p) % a.world;  // stagger destinations across ranks
          reinterpret_cast<float4*>(h.data[q])[i] = pv;
          if (h.shadow[q]) reinterpret_cast<uint2*>(h.shadow[q])[i] = s;
        }
      }
    }
  }
  if (!meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err)) return;
  clear_local_grads(h, a, sh);
}

// ------------------------------------------------------------------ clip mode
// Bucket launch: average shard r of the bucket in place (this rank's own
// gradient buffer holds the result) and add its sum of squares to *a.sumsq.
// No end meeting: the shard-r elements are touched by rank r only, and the
// peers' gradients are cleared by the apply launch, which follows this one on
// every rank's stream.
template <int W>
__global__ void __launch_bounds__(512, 2) reduce_scatter_kernel(const __grid_constant__ FusedArgs a,
                                                 const __grid_constant__ Handles h) {
  constexpr int ILP = IlpFor<W>::value;
  __shared__ float red[32];
  if (!meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err)) return;
  const Shard sh(a);
  const int64_t lo = sh.s0(a.rank), hi = sh.s1(a.rank);
  const float gs = grad_scale(a);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float ss = 0.f;
  for (int64_t i0 = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < hi;
       i0 += ILP * stride) {
    int64_t idx[ILP];
    bool live[ILP];
#pragma unroll
    for (int j = 0; j < ILP; ++j) {
      idx[j] = i0 + j * stride;
      live[j] = idx[j] < hi;
    }
    float4 g[ILP];
    gather_sum<W, ILP>(h, a.world, idx, live, g);
#pragma unroll
    for (int j = 0; j < ILP; ++j) {
      if (!live[j]) break;
      scale4(g[j], gs);
      ss += dot4(g[j]);
      reinterpret_cast<float4*>(h.grad[a.rank])[idx[j]] = g[j];
    }
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0 && a.sumsq) atomicAdd(a.sumsq, ss);
}

// Apply launch: publish this rank's sum of squares, meet, derive the global
// norm and the clip coefficient (max_norm / (norm + 1e-6) when the norm
// exceeds max_norm), update shard r of every bucket of the table, all-gather
// the weights, clear every local gradient, meet again.
template <class U>
__global__ void __launch_bounds__(512) clip_apply_kernel(const __grid_constant__ FusedArgs a,
                                                 const __grid_constant__ Handles h) {
  uint32_t* sig = h.sig[a.rank];
  __shared__ float local_ss;
  if (threadIdx.x == 0) {
    local_ss = *reinterpret_cast<volatile float*>(a.sumsq);
    __threadfence();
    // the last block to read the accumulator resets it for the next step
    const uint32_t n = atomicAdd(sig + SigLayout::kCount + a.bucket, 1u);
    if (n == gridDim.x - 1) {
      *a.sumsq = 0.f;
      sig[SigLayout::kCount + a.bucket] = 0u;
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < a.world)
    h.sig[threadIdx.x][SigLayout::kMass + (a.bucket * kMaxRanks + a.rank) * 2] =
        __float_as_uint(local_ss);
  if (!meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err)) return;
  float total = 0.f;
  for (int p = 0; p < a.world; ++p)
    total += __uint_as_float(ld_acquire_sys(sig + SigLayout::kMass + (a.bucket * kMaxRanks + p) * 2));
  const float norm = sqrtf(total);
  const float coef = (a.max_norm > 0.f && norm > a.max_norm) ? a.max_norm / (norm + 1e-6f) : 1.f;
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.norm_out) *a.norm_out = norm;
  const U upd(a);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  float4* gl = reinterpret_cast<float4*>(h.grad[a.rank]);
  for (int k = 0; k < a.nb; ++k) {
    FusedArgs ab = a;
    ab.start = a.table[2 * k];
    ab.end = a.table[2 * k + 1];
    const Shard sh(ab);
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < sh.per; j += stride) {
      for (int s = 0; s < a.world; ++s) {
        const int64_t i = sh.s0(s) + j;
        if (i >= sh.s1(s)) continue;
        if (s == a.rank) {
          float4 g = gl[i];
          scale4(g, coef);
          float4 pv = reinterpret_cast<const float4*>(h.data[a.rank])[i];
          upd(pv, g, i);
          const uint2 sb = bf16x4(pv);
          for (int p = 0; p < a.world; ++p) {
            const int q = (a.rank + p) % a.world;
            reinterpret_cast<float4*>(h.data[q])[i] = pv;
            if (h.shadow[q]) reinterpret_cast<uint2*>(h.shadow[q])[i] = sb;
          }
        }
        gl[i] = z;
      }
    }
  }
  meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err);
}

// ------------------------------------------------------------------ plain all-reduce
// In place over h.grad. Two-shot: rank r reduces shard r from every peer and
// writes the result into every peer's shard r (only rank r touches shard r).
// One-shot: every rank reduces the whole range into its data region (scratch),
// meets, and copies it into its gradient buffer.
template <int W>
__global__ void __launch_bounds__(512, 2) all_reduce_kernel(const __grid_constant__ FusedArgs a,
                                                 const __grid_constant__ Handles h) {
  constexpr int ILP = IlpFor<W>::value;
  if (!meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err)) return;
  const Shard sh(a);
  const int64_t lo = a.oneshot ? sh.b0 : sh.s0(a.rank);
  const int64_t hi = a.oneshot ? sh.b1 : sh.s1(a.rank);
  const float sc = a.average ? 1.f / (float)a.world : 1.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < hi;
       i0 += ILP * stride) {
    int64_t idx[ILP];
    bool live[ILP];
#pragma unroll
    for (int j = 0; j < ILP; ++j) {
      idx[j] = i0 + j * stride;
      live[j] = idx[j] < hi;
    }
    float4 g[ILP];
    gather_sum<W, ILP>(h, a.world, idx, live, g);
#pragma unroll
    for (int j = 0; j < ILP; ++j) {
      if (!live[j]) break;
      scale4(g[j], sc);
      if (a.oneshot) {
        reinterpret_cast<float4*>(h.data[a.rank])[idx[j]] = g[j];
      } else {
        for (int p = 0; p < a.world; ++p) {
          const int q = (a.rank + p) % a.world;
          reinterpret_cast<float4*>(h.grad[q])[idx[j]] = g[j];
        }
      }
    }
  }
  if (!meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err)) return;
  if (a.oneshot) {
    const float4* src = reinterpret_cast<const float4*>(h.data[a.rank]);
    float4* dst = reinterpret_cast<float4*>(h.grad[a.rank]);
    for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi; i += stride)
      dst[i] = src[i];
  }
}

// ------------------------------------------------------------------ weighted average
// data <- sum_p (m_p / sum m) data_p over the parameter part and
// sum_p (mover_p / sum mover) data_p over the buffer part (elements at or past
// buf_start). Every rank publishes (m, mover) into every peer's mass slot of
// this launch before the start meeting. When no rank did any work (sum m == 0)
// nothing changes (the reference skips both reduces). Divergence: rank r
// computes, over shard r, sum (data_p - avg)^2 for every p and sum avg^2, and
// stores them into rank p's partial slots; after the end meeting each rank
// adds its partials into a.div.
__global__ void __launch_bounds__(512, 2) weighted_average_kernel(const __grid_constant__ FusedArgs a,
                                                 const __grid_constant__ Handles h) {
  uint32_t* sig = h.sig[a.rank];
  __shared__ float w_sh[kMaxRanks], wb_sh[kMaxRanks];
  __shared__ float red[32];
  __shared__ int skip_sh;
  if ((int)threadIdx.x < a.world) {
    uint32_t* dst = h.sig[threadIdx.x] + SigLayout::kMass + (a.bucket * kMaxRanks + a.rank) * 2;
    dst[0] = __float_as_uint(a.mass);
    dst[1] = __float_as_uint(a.mover);
  }
  if (!meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err)) return;
  if (threadIdx.x == 0) {
    float tot = 0.f, totb = 0.f;
    for (int p = 0; p < a.world; ++p) {
      const uint32_t* src = sig + SigLayout::kMass + (a.bucket * kMaxRanks + p) * 2;
      w_sh[p] = fmaxf(__uint_as_float(ld_acquire_sys(src)), 0.f);
      wb_sh[p] = fmaxf(__uint_as_float(ld_acquire_sys(src + 1)), 0.f);
      tot += w_sh[p];
      totb += wb_sh[p];
    }
    skip_sh = !(tot > 0.f);
    for (int p = 0; p < a.world; ++p) {
      w_sh[p] = tot > 0.f ? w_sh[p] / tot : 0.f;
      wb_sh[p] = totb > 0.f ? wb_sh[p] / totb : w_sh[p];
    }
  }
  __syncthreads();
  const Shard sh(a);
  const int64_t lo = sh.s0(a.rank), hi = sh.s1(a.rank);
  const int64_t bstart = a.buf_start >= 0 ? a.buf_start / 4 : sh.b1;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float d2[kMaxRanks];
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p) d2[p] = 0.f;
  float p2 = 0.f;
  if (!skip_sh) {
    for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi; i += stride) {
      const bool is_buf = i >= bstart;
      float4 x[kMaxRanks];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < a.world) x[p] = ld_cg4(h.data[p] + 4 * i);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p) {
        if (p < a.world) {
          const float w = is_buf ? wb_sh[p] : w_sh[p];
          acc.x += w * x[p].x; acc.y += w * x[p].y; acc.z += w * x[p].z; acc.w += w * x[p].w;
        }
      }
      if (!is_buf) {
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p) {
          if (p < a.world) {
            const float4 d = make_float4(x[p].x - acc.x, x[p].y - acc.y, x[p].z - acc.z,
                                         x[p].w - acc.w);
            d2[p] += dot4(d);
          }
        }
        p2 += dot4(acc);
      }
      const uint2 s = bf16x4(acc);
      for (int p = 0; p < a.world; ++p) {
        const int q = (a.rank + p) % a.world;
        reinterpret_cast<float4*>(h.data[q])[i] = acc;
        if (h.shadow[q]) reinterpret_cast<uint2*>(h.shadow[q])[i] = s;
      }
    }
  }
  if (a.div) {
    // partials for every rank p: (sum over shard r of (data_p - avg)^2, sum avg^2)
    __shared__ float part_sh[kMaxRanks][2];
    for (int p = 0; p < a.world; ++p) {
      const float v = block_sum(d2[p], red);
      if (threadIdx.x == 0) part_sh[p][0] = v;
    }
    const float pp = block_sum(p2, red);
    if (threadIdx.x == 0)
      for (int p = 0; p < a.world; ++p) part_sh[p][1] = pp;
    __syncthreads();
    if ((int)threadIdx.x < a.world) {
      const int p = threadIdx.x;
      uint32_t* dst = h.sig[p] + SigLayout::kPart + (blockIdx.x * kMaxRanks + a.rank) * 2;
      dst[0] = __float_as_uint(part_sh[p][0]);
      dst[1] = __float_as_uint(part_sh[p][1]);
    }
  }
  if (!meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err)) return;
  if (a.div && threadIdx.x == 0) {
    float dd = 0.f, pp = 0.f;
    for (int p = 0; p < a.world; ++p) {
      const uint32_t* src = sig + SigLayout::kPart + (blockIdx.x * kMaxRanks + p) * 2;
      dd += __uint_as_float(ld_acquire_sys(src));
      pp += __uint_as_float(ld_acquire_sys(src + 1));
    }
    atomicAdd(a.div, dd);
    atomicAdd(a.div + 1, pp);
  }
}

// ------------------------------------------------------------------ broadcast pull
__global__ void __launch_bounds__(512) broadcast_pull_kernel(const __grid_constant__ FusedArgs a,
                                                 const __grid_constant__ Handles h) {
  if (!meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err)) return;
  const Shard sh(a);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (a.rank != a.root) {
    const float4* src = reinterpret_cast<const float4*>(h.data[a.root]);
    float4* dst = reinterpret_cast<float4*>(h.data[a.rank]);
    uint2* shd = reinterpret_cast<uint2*>(h.shadow[a.rank]);
    for (int64_t i0 = sh.b0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < sh.b1;
         i0 += kIlp * stride) {
      float4 v[kIlp];
#pragma unroll
      for (int j = 0; j < kIlp; ++j) {
        const int64_t i = i0 + j * stride;
        v[j] = i < sh.b1 ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < kIlp; ++j) {
        const int64_t i = i0 + j * stride;
        if (i < sh.b1) {
          dst[i] = v[j];
          if (shd) shd[i] = bf16x4(v[j]);
        }
      }
    }
  } else if (h.shadow[a.rank]) {
    // the root refreshes its own shadow so every rank ends with the same bits
    const float4* src = reinterpret_cast<const float4*>(h.data[a.rank]);
    uint2* shd = reinterpret_cast<uint2*>(h.shadow[a.rank]);
    for (int64_t i = sh.b0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < sh.b1; i += stride)
      shd[i] = bf16x4(src[i]);
  }
  // the root must not change its buffer until everyone has pulled
  meet(h, a.rank, a.world, a.bucket, a.timeout_ns, a.err);
}

// Kernel selection by world size: 2, 4 and 8 ranks get the compile-time
// gather (every peer's loads in flight at once), other sizes the generic one.
struct ArAdamWK {
  template <int W> static const void* fn() { return (const void*)ar_update_kernel<AdamWUpdate, W>; }
};
struct ArSgdK {
  template <int W> static const void* fn() { return (const void*)ar_update_kernel<SgdUpdate, W>; }
};
struct AllReduceK {
  template <int W> static const void* fn() { return (const void*)all_reduce_kernel<W>; }
};
struct ReduceScatterK {
  template <int W> static const void* fn() { return (const void*)reduce_scatter_kernel<W>; }
};
template <class K>
const void* pick_world(int world, int* ilp) {
  switch (world) {
    case 2: *ilp = IlpFor<2>::value; return K::template fn<2>();
    case 4: *ilp = IlpFor<4>::value; return K::template fn<4>();
    case 8: *ilp = IlpFor<8>::value; return K::template fn<8>();
    default: *ilp = IlpFor<0>::value; return K::template fn<0>();
  }
}

}  // namespace

cudaError_t launch_fused(FusedOp op, const FusedArgs& a, const PeerPtrs& ptrs, cudaStream_t st) {
  if (a.world < 1 || a.world > kMaxRanks || a.rank < 0 || a.rank >= a.world || a.bucket < 0 ||
      a.bucket >= kMaxSlots)
    return cudaErrorInvalidValue;
  if ((a.start & 3) || (a.end & 3) || a.end < a.start) return cudaErrorInvalidValue;
  if (a.threads != 128 && a.threads != 256 && a.threads != 512) return cudaErrorInvalidValue;
  Handles h;
  for (int p = 0; p < kMaxRanks; ++p) {
    h.data[p] = p < a.world ? ptrs.data[p] : nullptr;
    h.grad[p] = p < a.world ? ptrs.grad[p] : nullptr;
    h.shadow[p] = p < a.world ? ptrs.shadow[p] : nullptr;
    h.sig[p] = p < a.world ? ptrs.sig[p] : nullptr;
  }
  const int threads = a.threads;
  const void* fn = nullptr;
  bool sharded = true;  // work per rank = one shard (false: the whole range)
  int ilp = IlpFor<0>::value;
  switch (op) {
    case FusedOp::kArAdamW: fn = pick_world<ArAdamWK>(a.world, &ilp); break;
    case FusedOp::kArSgd: fn = pick_world<ArSgdK>(a.world, &ilp); break;
    case FusedOp::kAllReduce: fn = pick_world<AllReduceK>(a.world, &ilp); break;
    case FusedOp::kWeightedAverage: fn = (const void*)weighted_average_kernel; break;
    case FusedOp::kBroadcast: fn = (const void*)broadcast_pull_kernel; sharded = false; break;
    case FusedOp::kReduceScatter: fn = pick_world<ReduceScatterK>(a.world, &ilp); break;
    case FusedOp::kClipApplyAdamW: fn = (const void*)clip_apply_kernel<AdamWUpdate>; break;
    case FusedOp::kClipApplySgd: fn = (const void*)clip_apply_kernel<SgdUpdate>; break;
  }
  if (fn == nullptr) return cudaErrorInvalidValue;
  if ((op == FusedOp::kArAdamW || op == FusedOp::kClipApplyAdamW) && (!a.m || !a.v || !a.lr || !a.step))
    return cudaErrorInvalidValue;
  if ((op == FusedOp::kArSgd || op == FusedOp::kClipApplySgd) && !a.lr) return cudaErrorInvalidValue;
  if ((op == FusedOp::kReduceScatter || op == FusedOp::kClipApplyAdamW ||
       op == FusedOp::kClipApplySgd) && !a.sumsq)
    return cudaErrorInvalidValue;
  if ((op == FusedOp::kClipApplyAdamW || op == FusedOp::kClipApplySgd) && (!a.table || a.nb <= 0))
    return cudaErrorInvalidValue;
  if (a.oneshot) sharded = false;
  // Blocks of a launch meet their counterparts on the peers, so the grid is
  // kept co-resident: capped by the occupancy of this kernel.
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int cap = std::min(kMaxBlocks, per_sm * num_sms());
  // default: enough blocks for kIlp float4 per thread of this rank's work
  int64_t work4 = (a.end - a.start) / 4;
  if (op == FusedOp::kClipApplyAdamW || op == FusedOp::kClipApplySgd) work4 = 1 << 30;
  if (sharded) work4 = (work4 + a.world - 1) / a.world;
  const int64_t want = std::max<int64_t>(1, (work4 + (int64_t)threads * ilp - 1) / ((int64_t)threads * ilp));
  // an explicit grid is an upper bound: small messages keep few blocks
  const int64_t lim = a.blocks > 0 ? std::min(a.blocks, cap) : cap;
  const int blocks = (int)std::min<int64_t>(want, lim);
  void* args[] = {(void*)&a, (void*)&h};
  cudaError_t e = cudaLaunchKernel(fn, dim3(blocks), dim3(threads), args, 0, st);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

int signal_words() { return SigLayout::kWords; }

}  // namespace flodl
