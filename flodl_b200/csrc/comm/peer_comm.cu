// Peer-memory communicator for one NVLink/NVSwitch node, and the fused
// collective kernels that run over it.
//
// Symmetric memory: every rank cudaMalloc's the same-sized regions (parameter
// arena, gradient arena, bf16 shadow arena, signal words) and exports CUDA IPC
// handles; each rank opens its peers' handles, so a kernel on rank r can load
// from / store to any rank's region over NVLink. NCCL (or the torch.distributed
// store) is only used to exchange the handles.
//
// Kernels (all spin-waits are bounded by %globaltimer; on expiry they record
// an error code in host-mapped memory and return):
//
//  fused_ar_adamw / fused_ar_sgd   per DDP bucket, the reference's
//      "all_reduce_gradients (Avg) then optimizer.step()" (flodl/src/distributed/
//      ddp.rs:249-260 + nn/optim/adam.rs:183-245) as ONE launch:
//        1. every block announces "rank r reached bucket k" on all peers
//        2. rank r reduce-scatters: sums shard r of the bucket's gradients
//           from all peers by peer loads (scaled by 1/world)
//        3. applies AdamW / SGD-momentum to its shard
//        4. stores the updated f32 weights and their bf16 shadow into every
//           peer's arenas (all-gather by peer stores)
//        5. counts completion on every peer; waits until all peers' shards
//           landed locally, then zeroes its local gradient bucket
//  weighted_average   cluster parameter averaging (ElChe NCCL modes,
//      worker/sync.rs:130-236): out = sum_i (n_i^gamma / sum_j n_j^gamma) W_i
//      with the count exchange folded into the signal words.
//  broadcast_pull     initial parameter broadcast: every rank pulls rank 0's
//      buffer (rank_entry.rs:619-623).
//  all_reduce         plain sum/avg all-reduce of a symmetric buffer (sweeps).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>

#include "../kernels/sm100_ptx.cuh"
#include "peer_comm.h"

namespace flodl {

namespace {

constexpr int kIlp = 2;  // float4 elements per thread and loop iteration

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float4 ld_cg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

// Wait until *p >= target (wrap-safe) or the deadline passes.
__device__ __forceinline__ bool wait_ge(const uint32_t* p, uint32_t target, uint64_t limit_ns,
                                        uint32_t* err, uint32_t code) {
  uint64_t t0 = 0;
  uint32_t spins = 0;
  while ((int32_t)(ld_acquire_sys(p) - target) < 0) {
    if ((++spins & 255u) == 0u) {
      if (t0 == 0) t0 = global_timer_ns();
      else if (global_timer_ns() - t0 > limit_ns) {
        if (err) atomicCAS_system(err, 0u, code);
        return false;
      }
    }
  }
  return true;
}

// Signal layout (u32 words of the symmetric signal region):
//   [ready  + k*kMaxRanks + src] : epoch at which rank src reached bucket k
//   [done   + k]                 : completion counter of bucket k (peers add)
//   [epoch  + k]                 : local: completed launches of bucket k
//   [finish + k]                 : local: blocks finished in the current launch
//   [base + k]                   : local: value of done[k] when the previous launch ended
// The completion target of a launch is base + world * gridDim, so launches of
// one slot may use different grid sizes.
struct SigLayout {
  static constexpr int kReady = 0;
  static constexpr int kDone = kReady + kMaxBuckets * kMaxRanks;
  static constexpr int kEpoch = kDone + kMaxBuckets;
  static constexpr int kFinish = kEpoch + kMaxBuckets;
  static constexpr int kCount = kFinish + kMaxBuckets;  // count/mass exchange (f32 bits)
  static constexpr int kBase = kCount + kMaxBuckets * kMaxRanks * 2;
  static constexpr int kGo = kBase + kMaxBuckets;       // local: all peers ready (epoch)
  static constexpr int kFinCnt = kGo + kMaxBuckets;     // local: blocks done with a phase
  static constexpr int kFinGo = kFinCnt + kMaxBuckets;  // local: phase complete everywhere
  static constexpr int kWords = kFinGo + kMaxBuckets;
};

struct Handles {
  float* data[kMaxRanks];
  float* grad[kMaxRanks];
  __nv_bfloat16* shadow[kMaxRanks];
  uint32_t* sig[kMaxRanks];
};

// Start-of-launch handshake. Only block 0 of each rank talks to the peers: it
// publishes "rank r reached this launch of slot k" on every peer and waits
// until every peer did the same, then opens a local gate that the other
// blocks of the launch wait on. Returns the launch epoch (1, 2, ... per slot).
__device__ __forceinline__ uint32_t announce(const Handles& h, int rank, int world, int bucket,
                                             uint32_t* sig_local) {
  __shared__ uint32_t epoch_sh;
  if (threadIdx.x == 0) {
    const uint32_t e = *(volatile uint32_t*)(sig_local + SigLayout::kEpoch + bucket) + 1;
    epoch_sh = e;
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int p = 0; p < world; ++p)
        st_release_sys(h.sig[p] + SigLayout::kReady + bucket * kMaxRanks + rank, e);
    }
  }
  __syncthreads();
  return epoch_sh;
}

__device__ __forceinline__ bool wait_all_ready(const Handles& h, int world, int bucket,
                                               uint32_t epoch, uint32_t* sig_local,
                                               uint64_t limit, uint32_t* err) {
  __shared__ int ok_sh;
  if (threadIdx.x == 0) {
    bool ok = true;
    if (blockIdx.x == 0) {
      for (int p = 0; p < world && ok; ++p)
        ok = wait_ge(sig_local + SigLayout::kReady + bucket * kMaxRanks + p, epoch, limit, err,
                     kErrPeerTimeout);
      if (ok) st_release_sys(sig_local + SigLayout::kGo + bucket, epoch);
    } else {
      ok = wait_ge(sig_local + SigLayout::kGo + bucket, epoch, limit, err, kErrPeerTimeout);
    }
    ok_sh = ok;
  }
  __syncthreads();
  return ok_sh != 0;
}

// End-of-phase handshake on completion slot `slot` (the bucket, or bucket + 1
// for a second phase). Every block makes its peer-memory writes visible and
// counts itself; the last block of this rank signals each peer once and waits
// until all peers did, then opens a local gate for the other blocks. The
// completion target is base + world, base = the slot's count when the
// previous launch ended (recorded by end_launch).
__device__ __forceinline__ bool phase_done(const Handles& h, int world, int slot, uint32_t epoch,
                                           uint32_t* sig_local, uint64_t limit, uint32_t* err) {
  __shared__ int ok_sh;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t prev = atomicAdd(sig_local + SigLayout::kFinCnt + slot, 1u);
    bool ok;
    if (prev == gridDim.x - 1) {
      sig_local[SigLayout::kFinCnt + slot] = 0;
      __threadfence_system();
      for (int p = 0; p < world; ++p) red_add_release_sys(h.sig[p] + SigLayout::kDone + slot, 1u);
      const uint32_t target =
          *(volatile uint32_t*)(sig_local + SigLayout::kBase + slot) + (uint32_t)world;
      ok = wait_ge(sig_local + SigLayout::kDone + slot, target, limit, err, kErrPeerTimeout);
      if (ok) st_release_sys(sig_local + SigLayout::kFinGo + slot, epoch);
    } else {
      ok = wait_ge(sig_local + SigLayout::kFinGo + slot, epoch, limit, err, kErrPeerTimeout);
    }
    ok_sh = ok;
  }
  __syncthreads();
  return ok_sh != 0;
}

__device__ __forceinline__ bool finish_bucket(const Handles& h, int world, int bucket,
                                              uint32_t epoch, uint32_t* sig_local, uint64_t limit,
                                              uint32_t* err) {
  return phase_done(h, world, bucket, epoch, sig_local, limit, err);
}

// The last local block of a launch records the done counters (slot and
// slot + 1, which the all-reduce uses for its second round) as the base of
// the next launch, then advances the epoch. No peer can add to them before
// this rank announces its next launch.
__device__ __forceinline__ void end_launch(int bucket, uint32_t* sig_local) {
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(sig_local + SigLayout::kFinish + bucket, 1u);
    if (prev == gridDim.x - 1) {
      sig_local[SigLayout::kFinish + bucket] = 0;
      for (int k = bucket; k < bucket + 2 && k < kMaxBuckets; ++k)
        sig_local[SigLayout::kBase + k] = *(volatile uint32_t*)(sig_local + SigLayout::kDone + k);
      __threadfence();
      atomicAdd(sig_local + SigLayout::kEpoch + bucket, 1u);
    }
  }
}

__device__ __forceinline__ void adamw4(float4& p, float4 g, float4& m, float4& v, float lr,
                                       float b1, float b2, float eps, float wd, float bc1,
                                       float bc2s) {
  float* pp = &p.x;
  float* gg = &g.x;
  float* mm = &m.x;
  float* vv = &v.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mm[i] = b1 * mm[i] + (1.f - b1) * gg[i];
    vv[i] = b2 * vv[i] + (1.f - b2) * gg[i] * gg[i];
    const float denom = sqrtf(vv[i]) / bc2s + eps;
    pp[i] = pp[i] * (1.f - lr * wd) - (lr / bc1) * mm[i] / denom;
  }
}

// ------------------------------------------------------------------ fused AR + AdamW
__global__ void __launch_bounds__(512) fused_ar_adamw_kernel(FusedArgs a, Handles h) {
  uint32_t* sig = h.sig[a.rank];
  const uint32_t epoch = announce(h, a.rank, a.world, a.bucket, sig);
  const uint64_t limit = a.timeout_ns;
  if (!wait_all_ready(h, a.world, a.bucket, epoch, sig, limit, a.err)) {
    end_launch(a.bucket, sig);
    return;
  }
  // shard of this rank (in float4 units)
  const int64_t n4 = (a.end - a.start) / 4;
  const int64_t per = (n4 + a.world - 1) / a.world;
  const int64_t s0 = a.start / 4 + per * a.rank;
  const int64_t s1 = min(a.start / 4 + n4, s0 + per);
  const float lr = *a.lr;
  const float t = *a.step;
  const float bc1 = 1.f - powf(a.beta1, t);
  const float bc2s = sqrtf(1.f - powf(a.beta2, t));
  const float gs = (a.gscale ? *a.gscale : 1.f) / (float)a.world;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // two float4 per thread and iteration: all peer loads of both are issued
  // before any use, doubling the bytes in flight over NVLink
  for (int64_t i0 = s0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < s1;
       i0 += kIlp * stride) {
    float4 g[kIlp];
#pragma unroll
    for (int j = 0; j < kIlp; ++j) g[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int p = 0; p < a.world; ++p) {
#pragma unroll
      for (int j = 0; j < kIlp; ++j) {
        const int64_t i = i0 + j * stride;
        if (i < s1) {
          const float4 x = ld_cg4(h.grad[p] + 4 * i);
          g[j].x += x.x; g[j].y += x.y; g[j].z += x.z; g[j].w += x.w;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kIlp; ++j) {
      const int64_t i = i0 + j * stride;
      if (i >= s1) break;
      float4 gj = g[j];
      gj.x *= gs; gj.y *= gs; gj.z *= gs; gj.w *= gs;
      float4 pv = reinterpret_cast<float4*>(h.data[a.rank])[i];
      float4 m = reinterpret_cast<float4*>(a.m)[i];
      float4 v = reinterpret_cast<float4*>(a.v)[i];
      adamw4(pv, gj, m, v, lr, a.beta1, a.beta2, a.eps, a.wd, bc1, bc2s);
      reinterpret_cast<float4*>(a.m)[i] = m;
      reinterpret_cast<float4*>(a.v)[i] = v;
      uint2 sh;
      sh.x = pack_bf16x2(pv.x, pv.y);
      sh.y = pack_bf16x2(pv.z, pv.w);
      for (int p = 0; p < a.world; ++p) {
        const int q = (a.rank + p) % a.world;  // stagger destinations across ranks
        reinterpret_cast<float4*>(h.data[q])[i] = pv;
        reinterpret_cast<uint2*>(h.shadow[q])[i] = sh;
      }
    }
  }
  if (!finish_bucket(h, a.world, a.bucket, epoch, sig, limit, a.err)) {
    end_launch(a.bucket, sig);
    return;
  }
  // every peer has read our gradients and written its shard: clear the bucket
  float4* gl = reinterpret_cast<float4*>(h.grad[a.rank]);
  for (int64_t i = a.start / 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
       i < a.start / 4 + n4; i += stride)
    gl[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  end_launch(a.bucket, sig);
}

// ------------------------------------------------------------------ fused AR + SGD
__global__ void __launch_bounds__(512) fused_ar_sgd_kernel(FusedArgs a, Handles h) {
  uint32_t* sig = h.sig[a.rank];
  const uint32_t epoch = announce(h, a.rank, a.world, a.bucket, sig);
  const uint64_t limit = a.timeout_ns;
  if (!wait_all_ready(h, a.world, a.bucket, epoch, sig, limit, a.err)) {
    end_launch(a.bucket, sig);
    return;
  }
  const int64_t n4 = (a.end - a.start) / 4;
  const int64_t per = (n4 + a.world - 1) / a.world;
  const int64_t s0 = a.start / 4 + per * a.rank;
  const int64_t s1 = min(a.start / 4 + n4, s0 + per);
  const float lr = *a.lr;
  const bool first = a.first ? (*a.first != 0.f) : false;
  const float gs = (a.gscale ? *a.gscale : 1.f) / (float)a.world;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = s0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < s1;
       i0 += kIlp * stride) {
    float4 gv[kIlp];
#pragma unroll
    for (int jj = 0; jj < kIlp; ++jj) gv[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int p = 0; p < a.world; ++p) {
#pragma unroll
      for (int jj = 0; jj < kIlp; ++jj) {
        const int64_t i = i0 + jj * stride;
        if (i < s1) {
          const float4 x = ld_cg4(h.grad[p] + 4 * i);
          gv[jj].x += x.x; gv[jj].y += x.y; gv[jj].z += x.z; gv[jj].w += x.w;
        }
      }
    }
#pragma unroll
    for (int jj = 0; jj < kIlp; ++jj) {
      const int64_t i = i0 + jj * stride;
      if (i >= s1) break;
      float4 g = gv[jj];
      float4 pv = reinterpret_cast<float4*>(h.data[a.rank])[i];
      float* pp = &pv.x;
      float* gg = &g.x;
      float4 bv = a.m ? reinterpret_cast<float4*>(a.m)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      float* bb = &bv.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float d = gg[e] * gs + a.wd * pp[e];
        if (a.m) {
          bb[e] = first ? d : a.momentum * bb[e] + (1.f - a.dampening) * d;
          d = a.nesterov ? d + a.momentum * bb[e] : bb[e];
        }
        pp[e] -= lr * d;
      }
      if (a.m) reinterpret_cast<float4*>(a.m)[i] = bv;
      uint2 sh;
      sh.x = pack_bf16x2(pv.x, pv.y);
      sh.y = pack_bf16x2(pv.z, pv.w);
      for (int p = 0; p < a.world; ++p) {
        const int q = (a.rank + p) % a.world;
        reinterpret_cast<float4*>(h.data[q])[i] = pv;
        if (h.shadow[q]) reinterpret_cast<uint2*>(h.shadow[q])[i] = sh;
      }
    }
  }
  if (!finish_bucket(h, a.world, a.bucket, epoch, sig, limit, a.err)) {
    end_launch(a.bucket, sig);
    return;
  }
  float4* gl = reinterpret_cast<float4*>(h.grad[a.rank]);
  for (int64_t i = a.start / 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
       i < a.start / 4 + n4; i += stride)
    gl[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  end_launch(a.bucket, sig);
}

// ------------------------------------------------------------------ plain all-reduce
// In place over h.grad (the symmetric buffer): out = sum (or avg) over ranks.
__global__ void __launch_bounds__(512) all_reduce_kernel(FusedArgs a, Handles h) {
  uint32_t* sig = h.sig[a.rank];
  const uint32_t epoch = announce(h, a.rank, a.world, a.bucket, sig);
  const uint64_t limit = a.timeout_ns;
  if (!wait_all_ready(h, a.world, a.bucket, epoch, sig, limit, a.err)) {
    end_launch(a.bucket, sig);
    return;
  }
  const int64_t n4 = (a.end - a.start) / 4;
  const int64_t per = (n4 + a.world - 1) / a.world;
  const int64_t s0 = a.start / 4 + per * a.rank;
  const int64_t s1 = min(a.start / 4 + n4, s0 + per);
  const float sc = a.average ? 1.f / (float)a.world : 1.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // reduce into registers first, then a second barrier before writing so no
  // rank overwrites a shard another rank is still reading
  for (int64_t i0 = s0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < s1;
       i0 += kIlp * stride) {
    float4 g[kIlp];
#pragma unroll
    for (int j = 0; j < kIlp; ++j) g[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int p = 0; p < a.world; ++p) {
#pragma unroll
      for (int j = 0; j < kIlp; ++j) {
        const int64_t i = i0 + j * stride;
        if (i < s1) {
          const float4 x = ld_cg4(h.grad[p] + 4 * i);
          g[j].x += x.x; g[j].y += x.y; g[j].z += x.z; g[j].w += x.w;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kIlp; ++j) {
      const int64_t i = i0 + j * stride;
      if (i < s1) {
        float4 gj = g[j];
        gj.x *= sc; gj.y *= sc; gj.z *= sc; gj.w *= sc;
        reinterpret_cast<float4*>(h.data[a.rank])[i] = gj;  // staging (data region)
      }
    }
  }
  if (!finish_bucket(h, a.world, a.bucket, epoch, sig, limit, a.err)) {
    end_launch(a.bucket, sig);
    return;
  }
  // all reads done everywhere: broadcast the reduced shard back into every grad buffer
  for (int64_t i = s0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < s1; i += stride) {
    const float4 g = reinterpret_cast<const float4*>(h.data[a.rank])[i];
    for (int p = 0; p < a.world; ++p) {
      const int q = (a.rank + p) % a.world;
      reinterpret_cast<float4*>(h.grad[q])[i] = g;
    }
  }
  // second completion round on a separate slot (bucket + 1): every rank's
  // result is in every buffer before anyone reuses them
  phase_done(h, a.world, a.bucket + 1, epoch, sig, limit, a.err);
  end_launch(a.bucket, sig);
}

// ------------------------------------------------------------------ weighted average
// data <- sum_p w_p data_p with w_p = n_p^gamma / sum_q n_q^gamma, where each
// rank publishes its n (work count) through the signal words. Optionally also
// writes divergence partials sum((pre - post)^2), sum(post^2) into a.m[0..1].
__global__ void __launch_bounds__(512) weighted_average_kernel(FusedArgs a, Handles h) {
  uint32_t* sig = h.sig[a.rank];
  // publish my mass before announcing readiness
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    for (int p = 0; p < a.world; ++p)
      st_release_sys(h.sig[p] + SigLayout::kCount + a.bucket * kMaxRanks * 2 + a.rank,
                     __float_as_uint(a.mass));
  }
  __syncthreads();
  const uint32_t epoch = announce(h, a.rank, a.world, a.bucket, sig);
  const uint64_t limit = a.timeout_ns;
  if (!wait_all_ready(h, a.world, a.bucket, epoch, sig, limit, a.err)) {
    end_launch(a.bucket, sig);
    return;
  }
  __shared__ float w_sh[kMaxRanks];
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int p = 0; p < a.world; ++p) {
      const float n = __uint_as_float(ld_acquire_sys(sig + SigLayout::kCount + a.bucket * kMaxRanks * 2 + p));
      w_sh[p] = powf(fmaxf(n, 0.f), a.gamma);
      tot += w_sh[p];
    }
    for (int p = 0; p < a.world; ++p) w_sh[p] = tot > 0.f ? w_sh[p] / tot : 1.f / a.world;
  }
  __syncthreads();
  const int64_t n4 = (a.end - a.start) / 4;
  const int64_t per = (n4 + a.world - 1) / a.world;
  const int64_t s0 = a.start / 4 + per * a.rank;
  const int64_t s1 = min(a.start / 4 + n4, s0 + per);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float d2 = 0.f, p2 = 0.f;
  for (int64_t i = s0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < s1; i += stride) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < a.world; ++p) {
      const float4 x = ld_cg4(h.data[p] + 4 * i);
      const float w = w_sh[p];
      acc.x += w * x.x; acc.y += w * x.y; acc.z += w * x.z; acc.w += w * x.w;
    }
    reinterpret_cast<float4*>(h.grad[a.rank])[i] = acc;  // staging in the scratch region
  }
  if (!finish_bucket(h, a.world, a.bucket, epoch, sig, limit, a.err)) {
    end_launch(a.bucket, sig);
    return;
  }
  for (int64_t i = s0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < s1; i += stride) {
    const float4 g = reinterpret_cast<const float4*>(h.grad[a.rank])[i];
    const float4 pre = reinterpret_cast<const float4*>(h.data[a.rank])[i];
    d2 += (pre.x - g.x) * (pre.x - g.x) + (pre.y - g.y) * (pre.y - g.y) +
          (pre.z - g.z) * (pre.z - g.z) + (pre.w - g.w) * (pre.w - g.w);
    p2 += g.x * g.x + g.y * g.y + g.z * g.z + g.w * g.w;
    uint2 sh;
    sh.x = pack_bf16x2(g.x, g.y);
    sh.y = pack_bf16x2(g.z, g.w);
    for (int p = 0; p < a.world; ++p) {
      const int q = (a.rank + p) % a.world;
      reinterpret_cast<float4*>(h.data[q])[i] = g;
      if (h.shadow[q]) reinterpret_cast<uint2*>(h.shadow[q])[i] = sh;
    }
  }
  if (a.m) {  // divergence partials of this rank's shard
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      d2 += __shfl_xor_sync(0xffffffffu, d2, o);
      p2 += __shfl_xor_sync(0xffffffffu, p2, o);
    }
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(a.m, d2);
      atomicAdd(a.m + 1, p2);
    }
  }
  const int b2 = a.bucket + 1;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < a.world; ++p) red_add_release_sys(h.sig[p] + SigLayout::kDone + b2, 1u);
    wait_ge(sig + SigLayout::kDone + b2,
            *(volatile uint32_t*)(sig + SigLayout::kBase + b2) + (uint32_t)(a.world * gridDim.x),
            limit, a.err, kErrPeerTimeout);
  }
  __syncthreads();
  // the gradient arena served as staging for this rank's shard: clear it
  for (int64_t i = s0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < s1; i += stride)
    reinterpret_cast<float4*>(h.grad[a.rank])[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  end_launch(a.bucket, sig);
}

// ------------------------------------------------------------------ broadcast pull
__global__ void __launch_bounds__(512) broadcast_pull_kernel(FusedArgs a, Handles h) {
  uint32_t* sig = h.sig[a.rank];
  const uint32_t epoch = announce(h, a.rank, a.world, a.bucket, sig);
  const uint64_t limit = a.timeout_ns;
  if (!wait_all_ready(h, a.world, a.bucket, epoch, sig, limit, a.err)) {
    end_launch(a.bucket, sig);
    return;
  }
  const int64_t n4 = (a.end - a.start) / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (a.rank != a.root) {
    const float4* src = reinterpret_cast<const float4*>(h.data[a.root]);
    float4* dst = reinterpret_cast<float4*>(h.data[a.rank]);
    for (int64_t i = a.start / 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
         i < a.start / 4 + n4; i += stride) {
      const float4 v = __ldcg(src + i);
      dst[i] = v;
      if (h.shadow[a.rank]) {
        uint2 sh;
        sh.x = pack_bf16x2(v.x, v.y);
        sh.y = pack_bf16x2(v.z, v.w);
        reinterpret_cast<uint2*>(h.shadow[a.rank])[i] = sh;
      }
    }
  }
  // the root must not change its buffer until everyone has pulled
  finish_bucket(h, a.world, a.bucket, epoch, sig, limit, a.err);
  end_launch(a.bucket, sig);
}

}  // namespace

cudaError_t launch_fused(FusedOp op, const FusedArgs& a, const PeerPtrs& ptrs, cudaStream_t st) {
  if (a.world < 1 || a.world > kMaxRanks || a.bucket < 0 || a.bucket + 1 >= kMaxBuckets)
    return cudaErrorInvalidValue;
  if ((a.start & 3) || (a.end & 3) || a.end < a.start) return cudaErrorInvalidValue;
  Handles h;
  for (int p = 0; p < kMaxRanks; ++p) {
    h.data[p] = p < a.world ? ptrs.data[p] : nullptr;
    h.grad[p] = p < a.world ? ptrs.grad[p] : nullptr;
    h.shadow[p] = p < a.world ? ptrs.shadow[p] : nullptr;
    h.sig[p] = p < a.world ? ptrs.sig[p] : nullptr;
  }
  const int threads = a.threads;
  const void* fn = nullptr;
  switch (op) {
    case FusedOp::kArAdamW: fn = (const void*)fused_ar_adamw_kernel; break;
    case FusedOp::kArSgd: fn = (const void*)fused_ar_sgd_kernel; break;
    case FusedOp::kAllReduce: fn = (const void*)all_reduce_kernel; break;
    case FusedOp::kWeightedAverage: fn = (const void*)weighted_average_kernel; break;
    case FusedOp::kBroadcast: fn = (const void*)broadcast_pull_kernel; break;
  }
  if (fn == nullptr) return cudaErrorInvalidValue;
  // Every block waits (bounded) for all blocks of all ranks, so the grid must
  // be co-resident: cap it by the occupancy of this kernel (0 = the cap).
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int cap = per_sm * num_sms();
  // default: enough blocks for about two float4 pairs per thread of this
  // rank's shard (small messages: few blocks, less start/finish overhead)
  const int64_t shard4 = ((a.end - a.start) / 4 + a.world - 1) / a.world;
  const int64_t want = std::max<int64_t>(1, (shard4 + threads * kIlp * 2 - 1) / (threads * kIlp * 2));
  int blocks = a.blocks > 0 ? std::min(a.blocks, cap) : (int)std::min<int64_t>(want, cap);
  FusedArgs al = a;
  al.blocks = blocks;
  void* args[] = {(void*)&al, (void*)&h};
  cudaError_t e = cudaLaunchKernel(fn, dim3(blocks), dim3(threads), args, 0, st);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

int signal_words() { return SigLayout::kWords; }

}  // namespace flodl
