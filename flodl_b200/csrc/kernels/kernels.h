// Host launchers of the non-GEMM sm_100a kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_sm100.h"

namespace flodl {

// ------------------------------------------------------------- LayerNorm
struct LnFwdArgs {
  const void* x = nullptr;  // [rows, C] f32 or bf16
  bool x_bf16 = false;
  const float* gamma = nullptr;
  const float* beta = nullptr;
  __nv_bfloat16* y_bf16 = nullptr;
  float* y_f32 = nullptr;
  float* mean = nullptr;
  float* rstd = nullptr;
  int rows = 0, C = 0;
  float eps = 1e-5f;
};
struct LnBwdArgs {
  const __nv_bfloat16* dy = nullptr;
  const void* x = nullptr;
  bool x_bf16 = false;
  const float* mean = nullptr;
  const float* rstd = nullptr;
  const float* gamma = nullptr;
  const float* dres = nullptr;  // f32 [rows, C] added to dx
  float* dx_f32 = nullptr;
  __nv_bfloat16* dx_bf16 = nullptr;
  float* dgamma = nullptr;  // accumulated
  float* dbeta = nullptr;   // accumulated
  float* colsum = nullptr;  // accumulated sum over rows of dx
  int rows = 0, C = 0;
  float* partials = nullptr;  // scratch [3, partial_blocks, C] for the two-stage reduction
  int partial_blocks = 0;
  bool pre_add = false;  // true: normalise the gradient (dy + dres); false: dx += dres afterwards
};
cudaError_t launch_ln_fwd(const LnFwdArgs& a, cudaStream_t st);
cudaError_t launch_ln_bwd(const LnBwdArgs& a, cudaStream_t st);
// RMSNorm (rmsnorm.cu): y = x * rstd * w over the last dimension C; x/y/dy/dx
// f32 or bf16 (bf16 = true), w (nullable), rstd and dw (nullable, +=) f32;
// the backward's dw needs C <= 8192.
cudaError_t launch_rms_fwd(const void* x, bool bf16, const float* w, void* y, float* rstd,
                           int rows, int C, float eps, cudaStream_t st);
cudaError_t launch_rms_bwd(const void* dy, const void* x, bool bf16, const float* w,
                           const float* rstd, void* dx, float* dw, int rows, int C,
                           cudaStream_t st);
// Dropout (dropout.cu): y = x * keep / (1 - p), keep drawn from Philox-4x32-10
// on (element, offset) with the key seed; the same seed and offset give the
// same mask (the backward calls it on dy). x/y f32 or bf16, 0 <= p < 1.
cudaError_t launch_dropout(const void* x, void* y, bool bf16, int64_t n, float p, uint64_t seed,
                           uint64_t offset, cudaStream_t st);
// Max pooling over NCHW planes (pool.cu): kernel, stride, padding, dilation.
struct PoolGeo {
  int kh, kw, sh, sw, ph, pw, dh, dw;
};
// y [planes, Ho, Wo] and idx (flat in-plane index of each maximum, -1 for an
// empty window); the backward adds dy at idx into dx (zeroed by the caller).
cudaError_t launch_maxpool_fwd(const void* x, bool bf16, void* y, int32_t* idx, int planes, int H,
                               int W, int Ho, int Wo, const PoolGeo& g, cudaStream_t st);
cudaError_t launch_maxpool_bwd(const void* dy, bool bf16, const int32_t* idx, void* dx, int planes,
                               int H, int W, int Ho, int Wo, cudaStream_t st);
// GroupNorm (groupnorm.cu) over x [N, C, HW] contiguous, G groups (C % G == 0);
// x/y/dy/dx f32 or bf16, gamma/beta/dgamma/dbeta (nullable, += ) and the
// per-(sample, group) mean/rstd f32.
cudaError_t launch_gn_fwd(const void* x, bool bf16, const float* gamma, const float* beta,
                          void* y, float* mean, float* rstd, int N, int C, int HW, int G,
                          float eps, cudaStream_t st);
cudaError_t launch_gn_bwd(const void* dy, const void* x, bool bf16, const float* gamma,
                          const float* mean, const float* rstd, void* dx, float* dgamma,
                          float* dbeta, int N, int C, int HW, int G, cudaStream_t st);
cudaError_t launch_colsum(const void* m, bool bf16, float* out, int rows, int C, cudaStream_t st,
                          const float* scale = nullptr, int ld = 0);
// Two-stage (deterministic) column sum; partials is scratch [nblocks, C].
// Single-pass column sums: nblocks row slices, one atomic per column and
// slice into out (accumulating; optionally scaled by *scale).
cudaError_t launch_colsum_atomic(const void* m, bool bf16, float* out, int rows, int C,
                                 int nblocks, cudaStream_t st, const float* scale = nullptr);
cudaError_t launch_colsum2(const void* m, bool bf16, float* out, int rows, int C, float* partials,
                           int nblocks, cudaStream_t st, const float* scale = nullptr);
int colsum_partial_blocks(int rows);
int ln_bwd_partial_blocks(int rows);

// ------------------------------------------------------------- cross entropy
struct CeArgs {
  const __nv_bfloat16* logits = nullptr;  // [T, V] (row pitch ld)
  int ld = 0;
  const int64_t* targets = nullptr;       // [T]
  int T = 0, V = 0;
  int64_t ignore_index = -100;
  float smoothing = 0.f;
  const float* inv_count = nullptr;       // device scalar: 1 / #valid rows
  float* loss = nullptr;                  // device scalar, accumulated mean loss
  __nv_bfloat16* dlogits = nullptr;       // [T, V] gradient of the mean loss (nullable)
  int ld_d = 0;                           // row pitch of dlogits (0: V)
  uint32_t* err = nullptr;                // error word: kErrBadLabel for a target outside [0, V)
};
// inv_count = 1 / #rows whose target is in [0, V) (ignore_index and out-of-range
// targets do not count; an out-of-range target that is not ignore_index also
// records kErrBadLabel in *err).
cudaError_t launch_ce_count(const int64_t* targets, int T, int V, int64_t ignore_index,
                            float* inv_count, float* loss_zero, uint32_t* err, cudaStream_t st);
cudaError_t launch_softmax_ce(const CeArgs& a, cudaStream_t st);

// ------------------------------------------------------------- embedding
cudaError_t launch_embed_fwd(const int64_t* ids, const float* tok, const float* pos,
                             const int64_t* type_ids, const float* type_tab, float* out,
                             __nv_bfloat16* out_bf16, int T, int S, int C, int V,
                             cudaStream_t st);
cudaError_t launch_embed_bwd_atomic(const int64_t* ids, const float* dy, float* dtok, int T, int C,
                                    cudaStream_t st);
cudaError_t launch_pos_grad(const float* dy, float* dpos, int B, int S, int C, cudaStream_t st);
cudaError_t launch_onehot_bf16(const int64_t* ids, __nv_bfloat16* out, int T, int V,
                               cudaStream_t st);

// ------------------------------------------------------------- optimizers
struct AdamWArgs {
  float* p = nullptr;
  float* g = nullptr;
  float* m = nullptr;
  float* v = nullptr;
  __nv_bfloat16* shadow = nullptr;  // bf16 copy of p for the forward GEMMs (nullable)
  int64_t n = 0;
  const float* lr = nullptr;     // device scalar
  const float* step = nullptr;   // device scalar (already incremented)
  const float* gscale = nullptr; // device scalar multiplier on g (clip / 1/world), nullable
  float beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, wd = 0.f;
  bool decoupled = true;  // AdamW (true) vs Adam with L2 (false)
  bool zero_grad = false;
};
cudaError_t launch_adamw(const AdamWArgs& a, cudaStream_t st);

struct SgdArgs {
  float* p = nullptr;
  float* g = nullptr;
  float* buf = nullptr;  // momentum buffer (nullable when momentum == 0)
  __nv_bfloat16* shadow = nullptr;
  int64_t n = 0;
  const float* lr = nullptr;
  const float* gscale = nullptr;
  const float* first = nullptr;  // device scalar: 1 on the first step (buf = g)
  float momentum = 0.f, dampening = 0.f, wd = 0.f;
  bool nesterov = false;
  bool zero_grad = false;
};
cudaError_t launch_sgd(const SgdArgs& a, cudaStream_t st);

// Sum of squares of x[0..n) accumulated into *out (f32).
cudaError_t launch_sumsq(const float* x, int64_t n, float* out, cudaStream_t st);
// *coef = min(1, max_norm / (sqrt(*sumsq) + 1e-6)); also writes the norm.
cudaError_t launch_clip_coef(const float* sumsq, float max_norm, float* coef, float* norm,
                             cudaStream_t st);
cudaError_t launch_add_scalar(float* x, float v, cudaStream_t st);

// ------------------------------------------------------------- elementwise
cudaError_t launch_cast_f32_bf16(const float* x, __nv_bfloat16* y, int64_t n, cudaStream_t st);

}  // namespace flodl

namespace flodl {
// dh = dy * gelu'(h), all bf16 [n]
cudaError_t launch_gelu_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* h, __nv_bfloat16* dh,
                            int64_t n, cudaStream_t st);
// y = a * b elementwise, bf16 (e.g. dy * GELU' kept by a GELU epilogue)
cudaError_t launch_mul_bf16(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* y,
                            int64_t n, cudaStream_t st);
// y = gelu(x), dydx = gelu'(x), f32 (the epilogue math, for numerics tests)
cudaError_t launch_gelu_eval_f32(const float* x, float* y, float* dydx, int64_t n,
                                 cudaStream_t st);
// y = gelu(x) bf16 -> bf16
cudaError_t launch_gelu_fwd(const __nv_bfloat16* x, __nv_bfloat16* y, int64_t n, cudaStream_t st);
// ------------------------------------------------------------- conv / batch norm (conv.cu)
// Activations are NHWC bf16; a convolution is im2col -> tcgen05 GEMM (-> col2im).
// cols [N*Ho*Wo, k*k*C], column (kh*k + kw)*C + ci; C a multiple of 8
cudaError_t launch_im2col(const __nv_bfloat16* x, __nv_bfloat16* cols, int N, int H, int W, int C,
                          int k, int s, int p, cudaStream_t st);
// Rectangular kernels with per-axis stride and padding (1-D convolutions run
// as kh = 1).
struct ConvGeo {
  int kh, kw, sh, sw, ph, pw;
};
cudaError_t launch_im2col_geo(const __nv_bfloat16* x, __nv_bfloat16* cols, int N, int H, int W,
                              int C, const ConvGeo& g, cudaStream_t st);
// Batch-norm backward sums folded into the kernel that produces the gradient
// dz of a batch norm's output: ws[0:C] += sum dz, ws[C:2C] += sum dz * xhat
// with xhat = (x - mean) * rstd; the last block copies both to sums[0:2C],
// adds them to dbeta / dgamma (nullable) and zeroes ws and *ticket.
struct BnBwdSums {
  const __nv_bfloat16* x;
  const float* mean;
  const float* rstd;
  float* dgamma;
  float* dbeta;
  float* sums;
  float* ws;
  unsigned* ticket;
};
// With bn, dx (after add and mask) is the dz of that batch norm; C / 8 must
// divide 256.
cudaError_t launch_col2im_geo(const __nv_bfloat16* dcols, int ldc, __nv_bfloat16* dx,
                              const void* add, bool add_f32, const __nv_bfloat16* mask, int N,
                              int H, int W, int C, const ConvGeo& g, cudaStream_t st,
                              const BnBwdSums* bn = nullptr);
cudaError_t launch_col2im(const __nv_bfloat16* dcols, int ldc, __nv_bfloat16* dx, const void* add,
                          bool add_f32, const __nv_bfloat16* mask, int N, int H, int W, int C,
                          int k, int s, int p, cudaStream_t st);
// ws: 2C f32 zeros, ticket: one zero word; both are left zeroed for the next call.
cudaError_t launch_bn_stats(const __nv_bfloat16* x, int64_t M, int C, float eps, float momentum,
                            float* mean, float* rstd, float* run_mean, float* run_var, float* ws,
                            unsigned* ticket, cudaStream_t st);
cudaError_t launch_bn_apply(const __nv_bfloat16* x, int64_t M, int C, const float* mean,
                            const float* rstd, const float* gamma, const float* beta,
                            const __nv_bfloat16* identity, bool relu, __nv_bfloat16* y,
                            cudaStream_t st);
// Batch norm from statistics a GEMM epilogue accumulated (ws[0:C] = sum y,
// ws[C:2C] = sum y^2 over M rows): writes mean/rstd, updates the running
// statistics, applies (+ identity, ReLU) and leaves ws and *ticket zeroed.
cudaError_t launch_bn_apply_sums(const __nv_bfloat16* x, int64_t M, int C, float* ws,
                                 unsigned* ticket, float eps, float momentum, float* mean,
                                 float* rstd, float* run_mean, float* run_var, const float* gamma,
                                 const float* beta, const __nv_bfloat16* identity, bool relu,
                                 __nv_bfloat16* y, cudaStream_t st);
// sums: 2C f32 scratch (sum dz, sum dz*xhat); dz_out (nullable) receives the masked dy.
cudaError_t launch_bn_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* ymask,
                          const __nv_bfloat16* x, int64_t M, int C, const float* mean,
                          const float* rstd, const float* gamma, float* dgamma, float* dbeta,
                          float* sums, float* ws, unsigned* ticket, __nv_bfloat16* dx,
                          __nv_bfloat16* dz_out, cudaStream_t st);
// The elementwise half of launch_bn_bwd, for sums already reduced.
cudaError_t launch_bn_bwd_apply(const __nv_bfloat16* dy, const __nv_bfloat16* ymask,
                                const __nv_bfloat16* x, int64_t M, int C, const float* mean,
                                const float* rstd, const float* gamma, const float* sums,
                                __nv_bfloat16* dx, __nv_bfloat16* dz_out, cudaStream_t st);
cudaError_t launch_avgpool_fwd(const __nv_bfloat16* x, __nv_bfloat16* y, int N, int HW, int C,
                               cudaStream_t st);
cudaError_t launch_avgpool_bwd(const __nv_bfloat16* dy, int ld, __nv_bfloat16* dx, int N, int HW,
                               int C, cudaStream_t st);
cudaError_t launch_nchw_to_nhwc(const float* x, __nv_bfloat16* y, int N, int C, int HW, int Cp,
                                cudaStream_t st);
// One convolution of a network-wide weight pack / gradient unpack table.
struct ConvPackEntry {
  const float* w;          // f32 OIHW parameter [cout, cin, k, k]
  __nv_bfloat16* packed;   // bf16 [cout, k*k*cin_pad], column (kh*k + kw)*cin_pad + ci
  float* gacc;             // f32 [cout, k*k*cin_pad] gradient in packed order (zeroed on unpack)
  float* grad;             // f32 OIHW gradient (+=)
  int cout, cin, cin_pad, k;
};
cudaError_t launch_pack_conv_weights(const ConvPackEntry* table, int n, int max_elems,
                                     cudaStream_t st);
cudaError_t launch_unpack_conv_grads(const ConvPackEntry* table, int n, int max_elems,
                                     cudaStream_t st);
cudaError_t launch_cast_pad(const float* x, __nv_bfloat16* y, int rows, int cols, int ld,
                            cudaStream_t st);

}  // namespace flodl
