// Host interface of the tcgen05 GEMM engine (gemm_sm100.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace flodl {

enum GemmEpiFlags : int {
  kEpiGelu = 1,        // out = gelu(acc + bias); GELU'(acc + bias) -> aux (if aux != null)
  kEpiDGelu = 2,       // out = acc * aux   (aux = GELU' kept by the forward epilogue)
  kEpiAccumulate = 4,  // out(f32) += result (atomic, also used for split-K)
};

struct GemmEpilogue {
  void* out = nullptr;  // bf16 or f32, row pitch ld_out elements
  int ld_out = 0;
  int out_f32 = 0;
  const float* bias = nullptr;      // f32 [N] or null
  const float* residual = nullptr;  // f32 [M, ld_res] or null (added last)
  int ld_res = 0;
  void* aux = nullptr;  // bf16 [M, ld_aux]: GELU' out (gelu) / in (dgelu)
  int ld_aux = 0;
  int flags = 0;
  float alpha = 1.f;
  const float* alpha_ptr = nullptr;  // optional device scalar multiplied into alpha
  float* colsum = nullptr;  // f32 [N] or null: += column sums of the output (TMA-store path)
  float* colsumsq = nullptr;  // f32 [N] or null: += column sums of squares (batch-norm statistics)
};

struct GemmArgs {
  const void* A = nullptr;  // bf16
  const void* B = nullptr;  // bf16
  int M = 0, N = 0, K = 0;
  int lda = 0, ldb = 0;  // row pitch (elements) of the stored matrices
  bool a_mn = false;     // A stored [K, M]
  bool b_mn = false;     // B stored [K, N]
  int k_splits = 1;      // >1 requires kEpiAccumulate with f32 output
  int bn = 0;            // 0 = auto, 128 or 256
  GemmEpilogue ep;
  uint32_t* err = nullptr;  // device error word (nullable)
};

// Which host-side step rejected the last launch_gemm call of this thread ("" if none).
const char* gemm_failure_detail();
// Why the last make_tmap_bf16_2d call of this thread failed.
const char* tmap_failure_detail();
cudaError_t launch_gemm(const GemmArgs& g, cudaStream_t stream);
bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t ld, uint32_t box_inner, uint32_t box_outer);
int num_sms();
void set_wait_limit_ns(uint64_t ns);

// Count of kernels launched by this library (all launchers increment it).
void note_launch(int n = 1);
uint64_t launch_count();
void reset_launch_count();

// Host-mapped error word shared by the compute kernels (bounded waits write
// a nonzero KernelError code here instead of hanging). Readable without a sync.
uint32_t* default_err_word();
uint32_t read_kernel_error();
void clear_kernel_error();

}  // namespace flodl
