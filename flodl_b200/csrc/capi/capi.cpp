// C interface of the kernel library (declarations and conventions: flodl.h).
//
// Each entry point validates its arguments, launches through the same host
// launchers the torch bindings use, and turns a failure into a return code
// plus a thread-local message, the way the reference's shim returns an error
// string from every call (flodl-sys/shim.h).
#include "flodl.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <string>

#include "../kernels/flash_attn.h"
#include "../kernels/gemm_sm100.h"
#include "../kernels/kernels.h"

namespace {

std::string& last_error() {
  thread_local std::string msg;
  return msg;
}

int fail(int code, const char* fn, const char* what) {
  last_error() = std::string(fn) + ": " + what;
  return code;
}

// Launch result -> return code. A stale error of an unrelated earlier call is
// cleared before the launch (cudaGetLastError is per thread, not per call).
int cuda_result(const char* fn, cudaError_t e, const char* detail = nullptr) {
  if (e == cudaSuccess) {
    last_error().clear();
    return FLODL_OK;
  }
  std::string m = std::string(fn) + ": " + cudaGetErrorString(e);
  if (detail && *detail) m += std::string(" (") + detail + ")";
  last_error() = m;
  return (int)e;
}

cudaStream_t as_stream(flodl_stream s) { return reinterpret_cast<cudaStream_t>(s); }
void clear_stale() { (void)cudaGetLastError(); }

template <typename T>
const __nv_bfloat16* bf(const T* p) {
  return reinterpret_cast<const __nv_bfloat16*>(p);
}
template <typename T>
__nv_bfloat16* bfm(T* p) {
  return reinterpret_cast<__nv_bfloat16*>(p);
}

}  // namespace

#define FLODL_EXPORT extern "C" __attribute__((visibility("default")))
#define REQUIRE(cond, what)                                          \
  do {                                                               \
    if (!(cond)) return fail(FLODL_ERR_INVALID_ARGUMENT, __func__, what); \
  } while (0)

FLODL_EXPORT int flodl_abi_version(void) { return FLODL_ABI_VERSION; }

FLODL_EXPORT const char* flodl_last_error(void) { return last_error().c_str(); }

FLODL_EXPORT int flodl_device_sm_count(int* out) {
  REQUIRE(out != nullptr, "out is NULL");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    clear_stale();
    return fail(FLODL_ERR_NO_DEVICE, __func__, "no current CUDA device");
  }
  return cuda_result(__func__, cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev));
}

FLODL_EXPORT uint32_t flodl_kernel_error(void) { return flodl::read_kernel_error(); }
FLODL_EXPORT void flodl_clear_kernel_error(void) { flodl::clear_kernel_error(); }
FLODL_EXPORT uint64_t flodl_launch_count(void) { return flodl::launch_count(); }

FLODL_EXPORT void flodl_set_wait_limit_ns(uint64_t ns) {
  flodl::set_wait_limit_ns(ns);
  flodl::set_flash_wait_limit_ns(ns);
}

// ------------------------------------------------------------------ GEMM
FLODL_EXPORT int flodl_gemm_bf16(const flodl_gemm_desc* d, flodl_stream stream) {
  REQUIRE(d != nullptr, "desc is NULL");
  REQUIRE(d->A && d->B && d->out, "A, B and out are required");
  REQUIRE(d->M > 0 && d->N > 0 && d->K > 0, "M, N and K must be positive");
  REQUIRE(d->k_splits >= 1, "k_splits must be >= 1");
  REQUIRE(d->k_splits == 1 || ((d->flags & FLODL_GEMM_ACCUMULATE) && d->out_f32),
          "k_splits > 1 needs FLODL_GEMM_ACCUMULATE with an f32 output");
  REQUIRE(!(d->flags & FLODL_GEMM_DGELU) || d->aux, "FLODL_GEMM_DGELU needs aux");
  flodl::GemmArgs g;
  g.A = d->A;
  g.B = d->B;
  g.M = d->M;
  g.N = d->N;
  g.K = d->K;
  g.lda = d->lda;
  g.ldb = d->ldb;
  g.a_mn = d->a_trans != 0;
  g.b_mn = d->b_trans != 0;
  g.k_splits = d->k_splits;
  g.ep.out = d->out;
  g.ep.ld_out = d->ld_out;
  g.ep.out_f32 = d->out_f32;
  g.ep.bias = d->bias;
  g.ep.residual = d->residual;
  g.ep.ld_res = d->ld_res;
  g.ep.aux = d->aux;
  g.ep.ld_aux = d->ld_aux;
  g.ep.flags = d->flags;
  g.ep.alpha = d->alpha;
  clear_stale();
  const cudaError_t e = flodl::launch_gemm(g, as_stream(stream));
  return cuda_result(__func__, e, e == cudaSuccess ? nullptr : flodl::gemm_failure_detail());
}

// ------------------------------------------------------------------ LayerNorm
FLODL_EXPORT int flodl_layer_norm_fwd(const void* x, int x_bf16, const float* gamma,
                                      const float* beta, uint16_t* y_bf16, float* y_f32,
                                      float* mean, float* rstd, int rows, int C, float eps,
                                      flodl_stream stream) {
  REQUIRE(x && mean && rstd, "x, mean and rstd are required");
  REQUIRE(y_bf16 || y_f32, "at least one output (y_bf16 or y_f32) is required");
  REQUIRE(rows > 0 && C > 0, "rows and C must be positive");
  if (C % 4 != 0) return fail(FLODL_ERR_UNSUPPORTED, __func__, "C must be a multiple of 4");
  flodl::LnFwdArgs a;
  a.x = x;
  a.x_bf16 = x_bf16 != 0;
  a.gamma = gamma;
  a.beta = beta;
  a.y_bf16 = bfm(y_bf16);
  a.y_f32 = y_f32;
  a.mean = mean;
  a.rstd = rstd;
  a.rows = rows;
  a.C = C;
  a.eps = eps;
  clear_stale();
  return cuda_result(__func__, flodl::launch_ln_fwd(a, as_stream(stream)));
}

FLODL_EXPORT int flodl_layer_norm_bwd(const uint16_t* dy, const void* x, int x_bf16,
                                      const float* mean, const float* rstd, const float* gamma,
                                      const float* dres, float* dx_f32, uint16_t* dx_bf16,
                                      float* dgamma, float* dbeta, float* colsum, int rows, int C,
                                      flodl_stream stream) {
  REQUIRE(dy && x && mean && rstd, "dy, x, mean and rstd are required");
  REQUIRE(dx_f32 || dx_bf16, "at least one output (dx_f32 or dx_bf16) is required");
  REQUIRE(rows > 0 && C > 0, "rows and C must be positive");
  if (C % 4 != 0) return fail(FLODL_ERR_UNSUPPORTED, __func__, "C must be a multiple of 4");
  flodl::LnBwdArgs a;
  a.dy = bf(dy);
  a.x = x;
  a.x_bf16 = x_bf16 != 0;
  a.mean = mean;
  a.rstd = rstd;
  a.gamma = gamma;
  a.dres = dres;
  a.dx_f32 = dx_f32;
  a.dx_bf16 = bfm(dx_bf16);
  a.dgamma = dgamma;
  a.dbeta = dbeta;
  a.colsum = colsum;
  a.rows = rows;
  a.C = C;
  clear_stale();
  return cuda_result(__func__, flodl::launch_ln_bwd(a, as_stream(stream)));
}

// ------------------------------------------------------------------ attention
FLODL_EXPORT int flodl_flash_attn_fwd(const uint16_t* qkv, uint16_t* out, float* lse2,
                                      const uint8_t* key_pad, int B, int S, int H, int D,
                                      int causal, float scale, flodl_stream stream) {
  REQUIRE(qkv && out && lse2, "qkv, out and lse2 are required");
  REQUIRE(B > 0 && S > 0 && H > 0, "B, S and H must be positive");
  if (D != 64) return fail(FLODL_ERR_UNSUPPORTED, __func__, "head_dim must be 64");
  flodl::FlashArgs a;
  a.qkv = bf(qkv);
  a.out = bfm(out);
  a.lse2 = lse2;
  a.key_pad = key_pad;
  a.B = B;
  a.S = S;
  a.H = H;
  a.D = D;
  a.causal = causal != 0;
  a.scale = scale;
  clear_stale();
  return cuda_result(__func__, flodl::launch_flash_fwd(a, as_stream(stream)));
}

FLODL_EXPORT int flodl_flash_attn_bwd(const uint16_t* dout, const uint16_t* qkv,
                                      const uint16_t* out, const float* lse2, uint16_t* dqkv,
                                      float* delta, float* dq_acc, float* dbias,
                                      const uint8_t* key_pad, int B, int S, int H, int D,
                                      int causal, float scale, flodl_stream stream) {
  REQUIRE(dout && qkv && out && lse2 && dqkv, "dout, qkv, out, lse2 and dqkv are required");
  REQUIRE(delta, "scratch delta is required");
  REQUIRE(dq_acc || !flodl::flash_bwd_needs_dq_acc(S), "scratch dq_acc is required for S > 256");
  REQUIRE(B > 0 && S > 0 && H > 0, "B, S and H must be positive");
  if (D != 64) return fail(FLODL_ERR_UNSUPPORTED, __func__, "head_dim must be 64");
  flodl::FlashArgs a;
  a.qkv = bf(qkv);
  a.out = const_cast<__nv_bfloat16*>(bf(out));
  a.lse2 = const_cast<float*>(lse2);
  a.key_pad = key_pad;
  a.dout = bf(dout);
  a.dqkv = bfm(dqkv);
  a.delta = delta;
  a.dq_acc = dq_acc;
  a.dbias = dbias;
  a.B = B;
  a.S = S;
  a.H = H;
  a.D = D;
  a.causal = causal != 0;
  a.scale = scale;
  clear_stale();
  return cuda_result(__func__, flodl::launch_flash_bwd(a, as_stream(stream)));
}

// ------------------------------------------------------------------ loss
FLODL_EXPORT int flodl_softmax_cross_entropy(const uint16_t* logits, int ld,
                                             const int64_t* targets, int T, int V,
                                             int64_t ignore_index, float smoothing, float* loss,
                                             uint16_t* dlogits, float* inv_count,
                                             flodl_stream stream) {
  REQUIRE(logits && targets && loss && inv_count, "logits, targets, loss and inv_count are required");
  REQUIRE(T > 0 && V > 0 && ld >= V, "T and V must be positive and ld >= V");
  REQUIRE(smoothing >= 0.f && smoothing < 1.f, "smoothing must be in [0, 1)");
  const cudaStream_t st = as_stream(stream);
  clear_stale();
  cudaError_t e = flodl::launch_ce_count(targets, T, V, ignore_index, inv_count, loss,
                                         flodl::default_err_word(), st);
  if (e != cudaSuccess) return cuda_result(__func__, e);
  flodl::CeArgs a;
  a.logits = bf(logits);
  a.ld = ld;
  a.targets = targets;
  a.T = T;
  a.V = V;
  a.ignore_index = ignore_index;
  a.smoothing = smoothing;
  a.inv_count = inv_count;
  a.loss = loss;
  a.dlogits = bfm(dlogits);
  a.ld_d = V;
  a.err = flodl::default_err_word();
  return cuda_result(__func__, flodl::launch_softmax_ce(a, st));
}

// ------------------------------------------------------------------ embedding
FLODL_EXPORT int flodl_embedding_fwd(const int64_t* ids, const float* tok, const float* pos,
                                     const int64_t* type_ids, const float* type_tab, float* out,
                                     uint16_t* out_bf16, int T, int S, int C, int V,
                                     flodl_stream stream) {
  REQUIRE(ids && tok, "ids and tok are required");
  REQUIRE(out || out_bf16, "at least one output is required");
  REQUIRE(T > 0 && C > 0 && V > 0 && S > 0, "T, S, C and V must be positive");
  REQUIRE((type_ids == nullptr) == (type_tab == nullptr), "type_ids and type_tab go together");
  clear_stale();
  return cuda_result(__func__, flodl::launch_embed_fwd(ids, tok, pos, type_ids, type_tab, out,
                                                       bfm(out_bf16), T, S, C, V,
                                                       as_stream(stream)));
}

FLODL_EXPORT int flodl_embedding_bwd(const int64_t* ids, const float* dy, float* dtok, int T,
                                     int C, flodl_stream stream) {
  REQUIRE(ids && dy && dtok, "ids, dy and dtok are required");
  REQUIRE(T > 0 && C > 0, "T and C must be positive");
  clear_stale();
  return cuda_result(__func__, flodl::launch_embed_bwd_atomic(ids, dy, dtok, T, C,
                                                              as_stream(stream)));
}

// ------------------------------------------------------------------ optimizers
FLODL_EXPORT int flodl_adamw_step(float* p, float* g, float* m, float* v, uint16_t* shadow,
                                  int64_t n, const float* lr, const float* step,
                                  const float* gscale, float beta1, float beta2, float eps,
                                  float weight_decay, int decoupled, int zero_grad,
                                  flodl_stream stream) {
  REQUIRE(p && g && m && v && lr && step, "p, g, m, v, lr and step are required");
  REQUIRE(n >= 0, "n must be non-negative");
  flodl::AdamWArgs a;
  a.p = p;
  a.g = g;
  a.m = m;
  a.v = v;
  a.shadow = bfm(shadow);
  a.n = n;
  a.lr = lr;
  a.step = step;
  a.gscale = gscale;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.wd = weight_decay;
  a.decoupled = decoupled != 0;
  a.zero_grad = zero_grad != 0;
  clear_stale();
  return cuda_result(__func__, flodl::launch_adamw(a, as_stream(stream)));
}

FLODL_EXPORT int flodl_sgd_step(float* p, float* g, float* buf, uint16_t* shadow, int64_t n,
                                const float* lr, const float* gscale, const float* first,
                                float momentum, float dampening, float weight_decay, int nesterov,
                                int zero_grad, flodl_stream stream) {
  REQUIRE(p && g && lr, "p, g and lr are required");
  REQUIRE(n >= 0, "n must be non-negative");
  REQUIRE(momentum == 0.f || buf, "momentum needs buf");
  flodl::SgdArgs a;
  a.p = p;
  a.g = g;
  a.buf = buf;
  a.shadow = bfm(shadow);
  a.n = n;
  a.lr = lr;
  a.gscale = gscale;
  a.first = first;
  a.momentum = momentum;
  a.dampening = dampening;
  a.wd = weight_decay;
  a.nesterov = nesterov != 0;
  a.zero_grad = zero_grad != 0;
  clear_stale();
  return cuda_result(__func__, flodl::launch_sgd(a, as_stream(stream)));
}

FLODL_EXPORT int flodl_grad_sumsq(const float* x, int64_t n, float* sumsq, flodl_stream stream) {
  REQUIRE(x && sumsq, "x and sumsq are required");
  REQUIRE(n >= 0, "n must be non-negative");
  clear_stale();
  return cuda_result(__func__, flodl::launch_sumsq(x, n, sumsq, as_stream(stream)));
}

FLODL_EXPORT int flodl_clip_coef(const float* sumsq, float max_norm, float* coef, float* norm,
                                 flodl_stream stream) {
  REQUIRE(sumsq && coef, "sumsq and coef are required");
  REQUIRE(max_norm > 0.f, "max_norm must be positive");
  clear_stale();
  return cuda_result(__func__, flodl::launch_clip_coef(sumsq, max_norm, coef, norm,
                                                       as_stream(stream)));
}

// ------------------------------------------------------------------ elementwise
FLODL_EXPORT int flodl_gelu_fwd(const uint16_t* x, uint16_t* y, int64_t n, flodl_stream stream) {
  REQUIRE(x && y, "x and y are required");
  REQUIRE(n >= 0, "n must be non-negative");
  clear_stale();
  return cuda_result(__func__, flodl::launch_gelu_fwd(bf(x), bfm(y), n, as_stream(stream)));
}

FLODL_EXPORT int flodl_gelu_bwd(const uint16_t* dy, const uint16_t* x, uint16_t* dx, int64_t n,
                                flodl_stream stream) {
  REQUIRE(dy && x && dx, "dy, x and dx are required");
  REQUIRE(n >= 0, "n must be non-negative");
  clear_stale();
  return cuda_result(__func__, flodl::launch_gelu_bwd(bf(dy), bf(x), bfm(dx), n,
                                                      as_stream(stream)));
}

FLODL_EXPORT int flodl_cast_f32_bf16(const float* x, uint16_t* y, int64_t n, flodl_stream stream) {
  REQUIRE(x && y, "x and y are required");
  REQUIRE(n >= 0, "n must be non-negative");
  clear_stale();
  return cuda_result(__func__, flodl::launch_cast_f32_bf16(x, bfm(y), n, as_stream(stream)));
}

// ------------------------------------------------------------------ batch norm
FLODL_EXPORT int flodl_batch_norm_stats(const uint16_t* x, int64_t M, int C, float eps,
                                        float momentum, float* mean, float* rstd,
                                        float* running_mean, float* running_var, float* ws,
                                        uint32_t* ticket, flodl_stream stream) {
  REQUIRE(x && mean && rstd && ws && ticket, "x, mean, rstd, ws and ticket are required");
  REQUIRE(M > 0 && C > 0, "M and C must be positive");
  REQUIRE((running_mean == nullptr) == (running_var == nullptr),
          "running_mean and running_var go together");
  clear_stale();
  return cuda_result(__func__, flodl::launch_bn_stats(bf(x), M, C, eps, momentum, mean, rstd,
                                                      running_mean, running_var, ws,
                                                      reinterpret_cast<unsigned*>(ticket),
                                                      as_stream(stream)));
}

FLODL_EXPORT int flodl_batch_norm_apply(const uint16_t* x, int64_t M, int C, const float* mean,
                                        const float* rstd, const float* gamma, const float* beta,
                                        const uint16_t* identity, int relu, uint16_t* y,
                                        flodl_stream stream) {
  REQUIRE(x && mean && rstd && y, "x, mean, rstd and y are required");
  REQUIRE(M > 0 && C > 0, "M and C must be positive");
  clear_stale();
  return cuda_result(__func__, flodl::launch_bn_apply(bf(x), M, C, mean, rstd, gamma, beta,
                                                      bf(identity), relu != 0, bfm(y),
                                                      as_stream(stream)));
}
