// Host interface of the sm_100a flash attention kernels (flash_attn.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_sm100.h"

namespace flodl {

struct FlashArgs {
  const __nv_bfloat16* qkv = nullptr;  // [B*S, 3*H*D]
  __nv_bfloat16* out = nullptr;        // [B*S, H*D] (fwd output / bwd input O)
  float* lse2 = nullptr;               // [B, H, S] base-2 log-sum-exp
  const uint8_t* key_pad = nullptr;    // [B, S] nonzero = masked key (nullable)
  // backward
  const __nv_bfloat16* dout = nullptr; // [B*S, H*D]
  __nv_bfloat16* dqkv = nullptr;       // [B*S, 3*H*D]
  float* delta = nullptr;              // [B, H, S] scratch
  float* dq_acc = nullptr;             // [B*S, H*D] f32 scratch (only if flash_bwd_needs_dq_acc(S))
  float* dbias = nullptr;              // [3*H*D] f32: += column sums of dqkv (nullable)
  int B = 0, S = 0, H = 0, D = 0;
  bool causal = false;
  float scale = 1.f;
  uint32_t* err = nullptr;
};

cudaError_t launch_flash_fwd(const FlashArgs& a, cudaStream_t st);
cudaError_t launch_flash_bwd(const FlashArgs& a, cudaStream_t st);
// Whether the backward for sequence length S uses the f32 dQ accumulator
// (S > 256: key-tile kernel); for S <= 256 dQ stays in tensor memory.
bool flash_bwd_needs_dq_acc(int S);
void set_flash_wait_limit_ns(uint64_t ns);

}  // namespace flodl
