/* C interface of the flodl_b200 sm_100a kernel library.
 *
 * The reference (fab2s/floDl) reaches libtorch through a C shim of about 330
 * `extern "C"` functions (flodl-sys/shim.h) that a Rust crate binds; every
 * function returns NULL or an error string. This header is the same kind of
 * seam over this library's own kernels: plain C types, raw device pointers,
 * no torch or CUDA headers needed to include it, and every function reports
 * failure by return code plus a thread-local message (flodl_last_error), so
 * a Rust/C/C++ front end can bind it without a C++ compiler.
 *
 * Conventions
 *   - Pointers are device pointers on the current CUDA device unless stated.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - bf16 tensors are raw 16-bit bfloat16 words; f32 is IEEE float.
 *   - Return value: FLODL_OK (0) on success; a negative flodl_status for an
 *     argument the library rejects before launching; a positive value is a
 *     cudaError_t from the launch. flodl_last_error() then explains it.
 *   - Kernels never hang: every internal wait is bounded and records a code
 *     in a host-mapped word that flodl_kernel_error() reads without a sync.
 *   - Nothing here allocates device memory; callers pass every scratch
 *     buffer, sized as documented per function.
 *
 * Linking: the functions are exported from flodl_b200/_C*.so, which depends
 * on libtorch's shared libraries (torch/lib on the loader path). */
#ifndef FLODL_B200_C_API_H
#define FLODL_B200_C_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FLODL_ABI_VERSION 1

typedef enum flodl_status {
  FLODL_OK = 0,
  FLODL_ERR_INVALID_ARGUMENT = -1, /* null pointer, bad size, bad alignment */
  FLODL_ERR_UNSUPPORTED = -2,      /* shape the kernels do not cover (e.g. head_dim != 64) */
  FLODL_ERR_NO_DEVICE = -3         /* no current CUDA device */
} flodl_status;

/* Error codes the kernels record in the host-mapped error word. */
typedef enum flodl_kernel_error_code {
  FLODL_KERNEL_OK = 0,
  FLODL_KERNEL_WAIT_TIMEOUT = 1, /* a bounded mbarrier/TMEM wait gave up */
  FLODL_KERNEL_PEER_TIMEOUT = 2, /* a peer-memory meeting gave up */
  FLODL_KERNEL_BAD_ARGS = 3,     /* a kernel rejected its launch arguments */
  FLODL_KERNEL_BAD_LABEL = 4     /* a cross-entropy target outside [0, V) */
} flodl_kernel_error_code;

typedef void* flodl_stream;

/* ---------------------------------------------------------------- library */
int flodl_abi_version(void);
/* Message of the last failing call on this thread ("" if none). */
const char* flodl_last_error(void);
/* Multiprocessor count of the current device, into *out. */
int flodl_device_sm_count(int* out);
/* Kernel error word (flodl_kernel_error_code); readable without a sync. */
uint32_t flodl_kernel_error(void);
void flodl_clear_kernel_error(void);
/* Kernels this library launched since load (all entry points count). */
uint64_t flodl_launch_count(void);
/* Limit of every bounded wait inside the GEMM / attention kernels. */
void flodl_set_wait_limit_ns(uint64_t ns);

/* ---------------------------------------------------------------- GEMM
 * out[M, N] = epilogue(alpha * A' B'), tcgen05 tensor cores, f32 accumulate.
 *   A' = A [M, K] (row pitch lda), or A^T when a_trans (A stored [K, M]).
 *   B' = B^T with B [N, K] (row pitch ldb; a Linear weight), or B [K, N]
 *        when b_trans (B stored [K, N]).
 * Epilogue, in this order: + bias[N]; GELU (flags & FLODL_GEMM_GELU, writes
 * GELU'(pre) to aux when aux != NULL) or * aux (FLODL_GEMM_DGELU); +
 * residual[M, ld_res] (f32); out is bf16 or f32 (out_f32). With
 * FLODL_GEMM_ACCUMULATE the f32 out is added to (k_splits > 1 splits K).
 * Operands need 16-byte aligned bases and pitches that are multiples of 8. */
#define FLODL_GEMM_GELU 1
#define FLODL_GEMM_DGELU 2
#define FLODL_GEMM_ACCUMULATE 4

typedef struct flodl_gemm_desc {
  const void* A;
  const void* B;
  int M, N, K;
  int lda, ldb;
  int a_trans, b_trans;
  void* out;
  int ld_out;
  int out_f32;
  const float* bias;     /* f32 [N] or NULL */
  const float* residual; /* f32 [M, ld_res] or NULL */
  int ld_res;
  void* aux; /* bf16 [M, ld_aux] or NULL */
  int ld_aux;
  int flags;
  float alpha;
  int k_splits; /* 1 unless FLODL_GEMM_ACCUMULATE */
} flodl_gemm_desc;

int flodl_gemm_bf16(const flodl_gemm_desc* d, flodl_stream stream);

/* ---------------------------------------------------------------- LayerNorm
 * Forward over rows of x [rows, C] (f32 or bf16 per x_bf16): y = (x - mean)
 * * rstd * gamma + beta into y_bf16 and/or y_f32 (either may be NULL);
 * mean/rstd f32 [rows] are kept for the backward. gamma/beta may be NULL. */
int flodl_layer_norm_fwd(const void* x, int x_bf16, const float* gamma, const float* beta,
                         uint16_t* y_bf16, float* y_f32, float* mean, float* rstd, int rows,
                         int C, float eps, flodl_stream stream);
/* Backward: dx (f32 and/or bf16) from dy (bf16), plus the optional residual
 * gradient dres (f32, added to dx); dgamma, dbeta and colsum (sum over rows
 * of dx) are accumulated (+=) when not NULL. */
int flodl_layer_norm_bwd(const uint16_t* dy, const void* x, int x_bf16, const float* mean,
                         const float* rstd, const float* gamma, const float* dres, float* dx_f32,
                         uint16_t* dx_bf16, float* dgamma, float* dbeta, float* colsum, int rows,
                         int C, flodl_stream stream);

/* ---------------------------------------------------------------- attention
 * Flash attention over a packed projection qkv [B*S, 3*H*D] (bf16; Q, K, V of
 * head h at columns h*D, H*D + h*D, 2*H*D + h*D). out [B*S, H*D] bf16,
 * lse2 [B, H, S] f32 (base-2 log-sum-exp, kept for the backward). key_pad
 * [B, S] bytes, nonzero = masked key, or NULL. D must be 64. */
int flodl_flash_attn_fwd(const uint16_t* qkv, uint16_t* out, float* lse2, const uint8_t* key_pad,
                         int B, int S, int H, int D, int causal, float scale,
                         flodl_stream stream);
/* Backward into dqkv [B*S, 3*H*D] bf16. Scratch: delta f32 [B*H*S], dq_acc
 * f32 [B*S*H*D] (no initial contents needed; unused, and may be NULL, when
 * S <= 256: dQ then stays in tensor memory). dbias f32 [3*H*D] or NULL:
 * += column sums of dqkv (the packed projection's bias gradient). */
int flodl_flash_attn_bwd(const uint16_t* dout, const uint16_t* qkv, const uint16_t* out,
                         const float* lse2, uint16_t* dqkv, float* delta, float* dq_acc,
                         float* dbias, const uint8_t* key_pad, int B, int S, int H, int D,
                         int causal, float scale, flodl_stream stream);

/* ---------------------------------------------------------------- loss
 * Mean softmax cross-entropy over T rows of logits [T, V] (bf16, pitch ld):
 * *loss = mean over rows whose target is in [0, V); rows equal to
 * ignore_index do not count; a target outside [0, V) that is not
 * ignore_index is skipped and recorded as FLODL_KERNEL_BAD_LABEL. dlogits
 * [T, V] bf16 (may be NULL) receives d(loss)/dlogits. Scratch: inv_count,
 * one f32. Label smoothing in [0, 1). */
int flodl_softmax_cross_entropy(const uint16_t* logits, int ld, const int64_t* targets, int T,
                                int V, int64_t ignore_index, float smoothing, float* loss,
                                uint16_t* dlogits, float* inv_count, flodl_stream stream);

/* ---------------------------------------------------------------- embedding
 * out[t] = tok[ids[t]] + pos[t % S] (+ type_tab[type_ids[t]]), C columns;
 * out f32 and/or out_bf16 (either NULL). pos/type may be NULL. */
int flodl_embedding_fwd(const int64_t* ids, const float* tok, const float* pos,
                        const int64_t* type_ids, const float* type_tab, float* out,
                        uint16_t* out_bf16, int T, int S, int C, int V, flodl_stream stream);
/* dtok[ids[t]] += dy[t] (f32 atomics). */
int flodl_embedding_bwd(const int64_t* ids, const float* dy, float* dtok, int T, int C,
                        flodl_stream stream);

/* ---------------------------------------------------------------- optimizers
 * In-place fused updates over n f32 elements. lr and step are DEVICE scalars
 * (so a captured CUDA graph replays with new values); step is the 1-based
 * step count after the increment. gscale (device scalar or NULL) multiplies
 * the gradient (clip coefficient, 1/world). shadow (bf16 [n] or NULL) gets
 * the updated weights in bf16. zero_grad clears g after reading it. */
int flodl_adamw_step(float* p, float* g, float* m, float* v, uint16_t* shadow, int64_t n,
                     const float* lr, const float* step, const float* gscale, float beta1,
                     float beta2, float eps, float weight_decay, int decoupled, int zero_grad,
                     flodl_stream stream);
/* SGD with momentum; buf may be NULL when momentum == 0; first (device
 * scalar, nonzero on the first step) initialises buf to the gradient. */
int flodl_sgd_step(float* p, float* g, float* buf, uint16_t* shadow, int64_t n, const float* lr,
                   const float* gscale, const float* first, float momentum, float dampening,
                   float weight_decay, int nesterov, int zero_grad, flodl_stream stream);
/* *sumsq += sum x^2 (global-norm clipping, first half). */
int flodl_grad_sumsq(const float* x, int64_t n, float* sumsq, flodl_stream stream);
/* *coef = min(1, max_norm / (sqrt(*sumsq) + 1e-6)); *norm = sqrt(*sumsq). */
int flodl_clip_coef(const float* sumsq, float max_norm, float* coef, float* norm,
                    flodl_stream stream);

/* ---------------------------------------------------------------- elementwise */
int flodl_gelu_fwd(const uint16_t* x, uint16_t* y, int64_t n, flodl_stream stream);
/* dx = dy * gelu'(x) */
int flodl_gelu_bwd(const uint16_t* dy, const uint16_t* x, uint16_t* dx, int64_t n,
                   flodl_stream stream);
int flodl_cast_f32_bf16(const float* x, uint16_t* y, int64_t n, flodl_stream stream);

/* ---------------------------------------------------------------- batch norm (NHWC bf16)
 * Training statistics over M = N*H*W rows of C channels; running stats
 * updated with momentum. Scratch ws: 2*C f32 zeros and ticket: one u32 zero,
 * both left zeroed for the next call. */
int flodl_batch_norm_stats(const uint16_t* x, int64_t M, int C, float eps, float momentum,
                           float* mean, float* rstd, float* running_mean, float* running_var,
                           float* ws, uint32_t* ticket, flodl_stream stream);
/* y = relu?((x - mean) * rstd * gamma + beta (+ identity)) */
int flodl_batch_norm_apply(const uint16_t* x, int64_t M, int C, const float* mean,
                           const float* rstd, const float* gamma, const float* beta,
                           const uint16_t* identity, int relu, uint16_t* y, flodl_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* FLODL_B200_C_API_H */
