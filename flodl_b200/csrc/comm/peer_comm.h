// Host interface of the peer-memory communicator (peer_comm.cu, peer_alloc.cpp).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../kernels/gemm_sm100.h"

namespace flodl {

constexpr int kMaxRanks = 8;
constexpr int kMaxSlots = 128;    // signal slots (one per bucket / collective kind)
constexpr int kMaxBlocks = 1024;  // CTAs of one launch
constexpr int kMaxBuckets = kMaxSlots;

enum class FusedOp : int {
  kArAdamW = 0,          // gradient all-reduce (Avg) + AdamW on one bucket
  kArSgd = 1,            // gradient all-reduce (Avg) + SGD-momentum on one bucket
  kAllReduce = 2,        // in-place sum/avg all-reduce of grad[start:end)
  kWeightedAverage = 3,  // cluster parameter (+ f32 buffer) averaging over data[start:end)
  kBroadcast = 4,        // every rank pulls data[start:end) from `root`
  kReduceScatter = 5,    // clip mode: average grads into this rank's shard + sum of squares
  kClipApplyAdamW = 6,   // clip mode: global norm -> clip coefficient -> AdamW over all buckets
  kClipApplySgd = 7,     // clip mode: same with SGD-momentum
};

struct PeerPtrs {
  float* data[kMaxRanks];
  float* grad[kMaxRanks];
  __nv_bfloat16* shadow[kMaxRanks];
  uint32_t* sig[kMaxRanks];
};

struct FusedArgs {
  int rank = 0, world = 1, root = 0;
  int bucket = 0;              // signal slot, [0, kMaxSlots)
  int64_t start = 0, end = 0;  // element range in the arenas (multiples of 4)
  int blocks = 0;              // CTAs (0: sized to the message, capped by co-residency)
  int threads = 512;           // threads per CTA: 128/256 let a launch share SMs with compute
  bool oneshot = false;        // every rank reads the whole range from every peer (no all-gather)
  // optimizer state (local, full arena size) and hyper-parameters
  float* m = nullptr;
  float* v = nullptr;
  const float* lr = nullptr;
  const float* step = nullptr;
  const float* gscale = nullptr;
  const float* first = nullptr;
  float beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, wd = 0.f;
  float momentum = 0.f, dampening = 0.f;
  bool nesterov = false;
  bool average = true;
  // weighted average: this rank's gamma-mass n^gamma (0 for an idle rank) and
  // mover indicator; elements at or past buf_start are f32 buffers averaged
  // with mover / sum(mover) instead of mass / sum(mass)
  float mass = 1.f, mover = 1.f;
  int64_t buf_start = -1;  // -1: no buffer part
  float* div = nullptr;    // optional [2]: += ||pre - post||^2, ||post||^2 of this rank's params
  // clip mode
  float* sumsq = nullptr;              // local accumulator of the reduced shards' sum of squares
  float* norm_out = nullptr;           // optional: global gradient norm (written by the apply)
  float max_norm = 0.f;
  const int64_t* table = nullptr;      // device [nb][2] bucket ranges for the apply kernel
  int nb = 0;
  uint64_t timeout_ns = 10000000000ull;
  uint32_t* err = nullptr;  // host-mapped error word
};

cudaError_t launch_fused(FusedOp op, const FusedArgs& a, const PeerPtrs& ptrs, cudaStream_t st);
int signal_words();

}  // namespace flodl
