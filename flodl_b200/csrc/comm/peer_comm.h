// Host interface of the peer-memory communicator (peer_comm.cu, peer_alloc.cpp).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../kernels/gemm_sm100.h"

namespace flodl {

constexpr int kMaxRanks = 8;
constexpr int kMaxBuckets = 512;

enum class FusedOp : int {
  kArAdamW = 0,
  kArSgd = 1,
  kAllReduce = 2,
  kWeightedAverage = 3,
  kBroadcast = 4,
};

struct PeerPtrs {
  float* data[kMaxRanks];
  float* grad[kMaxRanks];
  __nv_bfloat16* shadow[kMaxRanks];
  uint32_t* sig[kMaxRanks];
};

struct FusedArgs {
  int rank = 0, world = 1, root = 0;
  int bucket = 0;          // signal slot (uses slots bucket and bucket+1)
  int64_t start = 0, end = 0;  // element range in the arenas (multiples of 4)
  int blocks = 0;           // CTAs (0: sized to the message, capped by co-residency)
  int threads = 512;        // threads per CTA: 128 lets a launch share SMs with compute kernels
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
  float mass = 1.f, gamma = 1.f;  // weighted average
  uint64_t timeout_ns = 10000000000ull;
  uint32_t* err = nullptr;  // host-mapped error word
};

cudaError_t launch_fused(FusedOp op, const FusedArgs& a, const PeerPtrs& ptrs, cudaStream_t st);
int signal_words();

}  // namespace flodl
