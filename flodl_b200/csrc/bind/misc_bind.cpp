// Torch bindings for LayerNorm, cross-entropy, embedding, optimizer and
// elementwise kernels.
#include "common.h"
#include "../kernels/kernels.h"

namespace {

using at::Tensor;
using c10::optional;

template <typename T>
T* ptr(const Tensor& t) { return reinterpret_cast<T*>(t.data_ptr()); }

void ln_fwd(const Tensor& x, const optional<Tensor>& gamma, const optional<Tensor>& beta,
            const optional<Tensor>& y_bf16, const optional<Tensor>& y_f32, const Tensor& mean,
            const Tensor& rstd, double eps) {
  FL_CHECK_CUDA(x);
  FL_CHECK(x.is_contiguous(), "x must be contiguous");
  const int C = (int)x.size(-1);
  const int rows = (int)(x.numel() / C);
  flodl::LnFwdArgs a;
  a.x = x.data_ptr();
  a.x_bf16 = x.scalar_type() == at::kBFloat16;
  FL_CHECK(a.x_bf16 || x.scalar_type() == at::kFloat, "x must be f32 or bf16");
  a.gamma = opt_ptr<const float>(gamma);
  a.beta = opt_ptr<const float>(beta);
  a.y_bf16 = opt_ptr<__nv_bfloat16>(y_bf16);
  a.y_f32 = opt_ptr<float>(y_f32);
  a.mean = ptr<float>(mean);
  a.rstd = ptr<float>(rstd);
  a.rows = rows;
  a.C = C;
  a.eps = (float)eps;
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_ln_fwd(a, cur_stream()));
}

// RMSNorm over the last dimension: y = x * rstd * w (x, y f32 or bf16).
void rms_fwd(const Tensor& x, const optional<Tensor>& w, Tensor& y, Tensor& rstd, double eps) {
  FL_CHECK_CUDA(x);
  FL_CHECK(x.is_contiguous() && y.is_contiguous() && y.scalar_type() == x.scalar_type() &&
               y.numel() == x.numel(), "rms_fwd: x, y contiguous, same dtype and size");
  const bool bf16 = x.scalar_type() == at::kBFloat16;
  FL_CHECK(bf16 || x.scalar_type() == at::kFloat, "rms_fwd: x must be f32 or bf16");
  const int C = (int)x.size(-1);
  const int rows = (int)(x.numel() / C);
  FL_CHECK(rstd.scalar_type() == at::kFloat && rstd.numel() >= rows, "rms_fwd: rstd [rows] f32");
  if (w) FL_CHECK(w->scalar_type() == at::kFloat && w->numel() == C, "rms_fwd: w [C] f32");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_rms_fwd(x.data_ptr(), bf16, opt_ptr<const float>(w), y.data_ptr(),
                                   ptr<float>(rstd), rows, C, (float)eps, cur_stream()));
}

void rms_bwd(const Tensor& dy, const Tensor& x, const optional<Tensor>& w, const Tensor& rstd,
             Tensor& dx, const optional<Tensor>& dw) {
  FL_CHECK_CUDA(x);
  FL_CHECK(dy.is_contiguous() && x.is_contiguous() && dx.is_contiguous() &&
               dy.scalar_type() == x.scalar_type() && dx.scalar_type() == x.scalar_type() &&
               dy.numel() == x.numel() && dx.numel() == x.numel(),
           "rms_bwd: dy, x, dx contiguous, same dtype and size");
  const int C = (int)x.size(-1);
  const int rows = (int)(x.numel() / C);
  if (dw) FL_CHECK(dw->scalar_type() == at::kFloat && dw->numel() == C, "rms_bwd: dw [C] f32");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_rms_bwd(dy.data_ptr(), x.data_ptr(), x.scalar_type() == at::kBFloat16,
                                   opt_ptr<const float>(w), ptr<float>(rstd), dx.data_ptr(),
                                   opt_ptr<float>(dw), rows, C, cur_stream()));
}

// GroupNorm over x [N, C, *] contiguous (f32 or bf16), G groups.
void gn_fwd(const Tensor& x, const optional<Tensor>& gamma, const optional<Tensor>& beta,
            Tensor& y, Tensor& mean, Tensor& rstd, int64_t G, double eps) {
  FL_CHECK_CUDA(x);
  FL_CHECK(x.dim() >= 2 && x.is_contiguous() && y.is_contiguous() &&
               y.scalar_type() == x.scalar_type() && y.numel() == x.numel(),
           "gn_fwd: x, y contiguous [N, C, *], same dtype and size");
  const bool bf16 = x.scalar_type() == at::kBFloat16;
  FL_CHECK(bf16 || x.scalar_type() == at::kFloat, "gn_fwd: x must be f32 or bf16");
  const int N = (int)x.size(0), Cc = (int)x.size(1);
  const int HW = (int)(x.numel() / ((int64_t)N * Cc));
  FL_CHECK(G > 0 && Cc % G == 0, "gn_fwd: C must divide into G groups");
  FL_CHECK(mean.numel() >= N * G && rstd.numel() >= N * G, "gn_fwd: mean/rstd [N*G] f32");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_gn_fwd(x.data_ptr(), bf16, opt_ptr<const float>(gamma),
                                  opt_ptr<const float>(beta), y.data_ptr(), ptr<float>(mean),
                                  ptr<float>(rstd), N, Cc, HW, (int)G, (float)eps, cur_stream()));
}

void gn_bwd(const Tensor& dy, const Tensor& x, const optional<Tensor>& gamma, const Tensor& mean,
            const Tensor& rstd, Tensor& dx, const optional<Tensor>& dgamma,
            const optional<Tensor>& dbeta, int64_t G) {
  FL_CHECK_CUDA(x);
  FL_CHECK(dy.is_contiguous() && x.is_contiguous() && dx.is_contiguous() &&
               dy.scalar_type() == x.scalar_type() && dx.scalar_type() == x.scalar_type() &&
               dy.numel() == x.numel() && dx.numel() == x.numel(),
           "gn_bwd: dy, x, dx contiguous, same dtype and size");
  const int N = (int)x.size(0), Cc = (int)x.size(1);
  const int HW = (int)(x.numel() / ((int64_t)N * Cc));
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_gn_bwd(dy.data_ptr(), x.data_ptr(), x.scalar_type() == at::kBFloat16,
                                  opt_ptr<const float>(gamma), ptr<float>(mean), ptr<float>(rstd),
                                  dx.data_ptr(), opt_ptr<float>(dgamma), opt_ptr<float>(dbeta), N,
                                  Cc, HW, (int)G, cur_stream()));
}

// Max pooling of x [planes, H, W] (f32 or bf16) into y [planes, Ho, Wo] with
// the argmax index per output (int32).
void maxpool_fwd(const Tensor& x, Tensor& y, Tensor& idx, int64_t kh, int64_t kw, int64_t sh,
                 int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw) {
  FL_CHECK_CUDA(x);
  FL_CHECK(x.is_contiguous() && y.is_contiguous() && idx.is_contiguous() && x.dim() >= 2 &&
               y.scalar_type() == x.scalar_type() && idx.scalar_type() == at::kInt &&
               idx.numel() == y.numel(),
           "maxpool_fwd: contiguous x, y (same dtype) and int32 idx like y");
  const bool bf16 = x.scalar_type() == at::kBFloat16;
  FL_CHECK(bf16 || x.scalar_type() == at::kFloat, "maxpool_fwd: x must be f32 or bf16");
  const int H = (int)x.size(-2), W = (int)x.size(-1);
  const int Ho = (int)y.size(-2), Wo = (int)y.size(-1);
  const int planes = (int)(x.numel() / ((int64_t)H * W));
  FL_CHECK(y.numel() == (int64_t)planes * Ho * Wo, "maxpool_fwd: y shape");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_maxpool_fwd(
      x.data_ptr(), bf16, y.data_ptr(), ptr<int32_t>(idx), planes, H, W, Ho, Wo,
      flodl::PoolGeo{(int)kh, (int)kw, (int)sh, (int)sw, (int)ph, (int)pw, (int)dh, (int)dw},
      cur_stream()));
}

void maxpool_bwd(const Tensor& dy, const Tensor& idx, Tensor& dx) {
  FL_CHECK_CUDA(dy);
  FL_CHECK(dy.is_contiguous() && idx.is_contiguous() && dx.is_contiguous() &&
               dy.scalar_type() == dx.scalar_type() && idx.numel() == dy.numel(),
           "maxpool_bwd: contiguous dy, dx (same dtype), idx like dy");
  const int H = (int)dx.size(-2), W = (int)dx.size(-1);
  const int Ho = (int)dy.size(-2), Wo = (int)dy.size(-1);
  const int planes = (int)(dx.numel() / ((int64_t)H * W));
  c10::cuda::CUDAGuard guard(dy.device());
  FL_CUDA_OK(flodl::launch_maxpool_bwd(dy.data_ptr(), dy.scalar_type() == at::kBFloat16,
                                       ptr<int32_t>(idx), dx.data_ptr(), planes, H, W, Ho, Wo,
                                       cur_stream()));
}

// Dropout with a counter-based mask (same seed and offset: same mask).
void dropout(const Tensor& x, Tensor& y, double p, int64_t seed, int64_t offset) {
  FL_CHECK_CUDA(x);
  FL_CHECK(x.is_contiguous() && y.is_contiguous() && y.scalar_type() == x.scalar_type() &&
               y.numel() == x.numel(), "dropout: x, y contiguous, same dtype and size");
  const bool bf16 = x.scalar_type() == at::kBFloat16;
  FL_CHECK(bf16 || x.scalar_type() == at::kFloat, "dropout: x must be f32 or bf16");
  FL_CHECK(p >= 0.0 && p < 1.0, "dropout: 0 <= p < 1");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_dropout(x.data_ptr(), y.data_ptr(), bf16, x.numel(), (float)p,
                                   (uint64_t)seed, (uint64_t)offset, cur_stream()));
}

void ln_bwd(const Tensor& dy, const Tensor& x, const Tensor& mean, const Tensor& rstd,
            const optional<Tensor>& gamma, const optional<Tensor>& dres,
            const optional<Tensor>& dx_f32, const optional<Tensor>& dx_bf16,
            const optional<Tensor>& dgamma, const optional<Tensor>& dbeta,
            const optional<Tensor>& colsum, bool pre_add) {
  FL_CHECK_CUDA(dy);
  FL_CHECK_BF16(dy);
  FL_CHECK(dy.is_contiguous() && x.is_contiguous(), "ln_bwd inputs must be contiguous");
  const int C = (int)x.size(-1);
  flodl::LnBwdArgs a;
  a.dy = ptr<__nv_bfloat16>(dy);
  a.x = x.data_ptr();
  a.x_bf16 = x.scalar_type() == at::kBFloat16;
  a.mean = ptr<float>(mean);
  a.rstd = ptr<float>(rstd);
  a.gamma = opt_ptr<const float>(gamma);
  a.dres = opt_ptr<const float>(dres);
  a.dx_f32 = opt_ptr<float>(dx_f32);
  a.dx_bf16 = opt_ptr<__nv_bfloat16>(dx_bf16);
  a.dgamma = opt_ptr<float>(dgamma);
  a.dbeta = opt_ptr<float>(dbeta);
  a.colsum = opt_ptr<float>(colsum);
  a.pre_add = pre_add;
  a.rows = (int)(x.numel() / C);
  a.C = C;
  c10::cuda::CUDAGuard guard(x.device());
  // column reductions (dgamma, dbeta, bias gradient) accumulate with one
  // atomic per column and block: no scratch, no second pass
  FL_CUDA_OK(flodl::launch_ln_bwd(a, cur_stream()));
}

void colsum(const Tensor& m, Tensor& out, const optional<Tensor>& scale) {
  FL_CHECK_CUDA(m);
  FL_CHECK_F32(out);
  const int C = (int)m.size(-1);
  c10::cuda::CUDAGuard guard(m.device());
  if (!m.is_contiguous()) {
    // row-strided 2-D view (e.g. the first V columns of a padded buffer)
    FL_CHECK(m.dim() == 2 && m.stride(1) == 1, "colsum input must be contiguous or a row-strided 2-D view");
    FL_CUDA_OK(flodl::launch_colsum(m.data_ptr(), m.scalar_type() == at::kBFloat16, ptr<float>(out),
                                    (int)m.size(0), C, cur_stream(), opt_ptr<const float>(scale),
                                    (int)m.stride(0)));
    return;
  }
  const int rows = (int)(m.numel() / C);
  const int nb = flodl::colsum_partial_blocks(rows);
  FL_CUDA_OK(flodl::launch_colsum_atomic(m.data_ptr(), m.scalar_type() == at::kBFloat16,
                                         ptr<float>(out), rows, C, nb, cur_stream(),
                                         opt_ptr<const float>(scale)));
}

// Returns nothing; writes loss (scalar, overwritten) and dlogits.
void softmax_ce(const Tensor& logits, const Tensor& targets, Tensor& loss, Tensor& inv_count,
                const optional<Tensor>& dlogits, int64_t ignore_index, double smoothing) {
  FL_CHECK_CUDA(logits);
  FL_CHECK_BF16(logits);
  FL_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D row-major");
  FL_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(), "targets must be int64");
  const int T = (int)logits.size(0), V = (int)logits.size(1);
  c10::cuda::CUDAGuard guard(logits.device());
  auto st = cur_stream();
  FL_CUDA_OK(flodl::launch_ce_count(ptr<int64_t>(targets), T, V, ignore_index,
                                    ptr<float>(inv_count), ptr<float>(loss), nullptr, st));
  flodl::CeArgs a;
  a.logits = ptr<__nv_bfloat16>(logits);
  a.ld = (int)logits.stride(0);
  a.targets = ptr<int64_t>(targets);
  a.T = T;
  a.V = V;
  a.ignore_index = ignore_index;
  a.smoothing = (float)smoothing;
  a.inv_count = ptr<float>(inv_count);
  a.loss = ptr<float>(loss);
  if (dlogits) {
    FL_CHECK(dlogits->dim() == 2 && dlogits->stride(1) == 1 && dlogits->size(0) == T &&
                 dlogits->size(1) == V,
             "dlogits must be [T, V] row-major (any row pitch)");
    a.dlogits = ptr<__nv_bfloat16>(*dlogits);
    a.ld_d = (int)dlogits->stride(0);
  }
  FL_CUDA_OK(flodl::launch_softmax_ce(a, st));
}

void embed_fwd(const Tensor& ids, const Tensor& tok, const optional<Tensor>& pos,
               const optional<Tensor>& type_ids, const optional<Tensor>& type_tab,
               const optional<Tensor>& out, const optional<Tensor>& out_bf16, int64_t S) {
  FL_CHECK_CUDA(ids);
  FL_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids must be int64");
  FL_CHECK_F32(tok);
  const int C = (int)tok.size(1), V = (int)tok.size(0);
  c10::cuda::CUDAGuard guard(ids.device());
  FL_CUDA_OK(flodl::launch_embed_fwd(ptr<int64_t>(ids), ptr<float>(tok), opt_ptr<float>(pos),
                                     opt_ptr<int64_t>(type_ids), opt_ptr<float>(type_tab),
                                     opt_ptr<float>(out), opt_ptr<__nv_bfloat16>(out_bf16),
                                     (int)ids.numel(), (int)S, C, V, cur_stream()));
}

void embed_bwd_atomic(const Tensor& ids, const Tensor& dy, Tensor& dtok) {
  c10::cuda::CUDAGuard guard(ids.device());
  FL_CHECK_F32(dy);
  FL_CUDA_OK(flodl::launch_embed_bwd_atomic(ptr<int64_t>(ids), ptr<float>(dy), ptr<float>(dtok),
                                            (int)ids.numel(), (int)dtok.size(1), cur_stream()));
}

void pos_grad(const Tensor& dy, Tensor& dpos, int64_t B, int64_t S) {
  c10::cuda::CUDAGuard guard(dy.device());
  FL_CHECK_F32(dy);
  FL_CUDA_OK(flodl::launch_pos_grad(ptr<float>(dy), ptr<float>(dpos), (int)B, (int)S,
                                    (int)dpos.size(1), cur_stream()));
}

void onehot_bf16(const Tensor& ids, Tensor& out) {
  c10::cuda::CUDAGuard guard(ids.device());
  FL_CUDA_OK(flodl::launch_onehot_bf16(ptr<int64_t>(ids), ptr<__nv_bfloat16>(out),
                                       (int)ids.numel(), (int)out.size(1), cur_stream()));
}

void adamw(Tensor& p, Tensor& g, Tensor& m, Tensor& v, const optional<Tensor>& shadow,
           const Tensor& lr, const Tensor& step, const optional<Tensor>& gscale, double beta1,
           double beta2, double eps, double wd, bool decoupled, bool zero_grad) {
  FL_CHECK_F32(p); FL_CHECK_F32(g); FL_CHECK_F32(m); FL_CHECK_F32(v);
  FL_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(),
           "adamw buffers must be contiguous");
  FL_CHECK(g.numel() == p.numel() && m.numel() == p.numel() && v.numel() == p.numel(), "adamw sizes");
  flodl::AdamWArgs a;
  a.p = ptr<float>(p); a.g = ptr<float>(g); a.m = ptr<float>(m); a.v = ptr<float>(v);
  if (shadow) { FL_CHECK_BF16(*shadow); FL_CHECK(shadow->numel() == p.numel(), "shadow size"); }
  a.shadow = opt_ptr<__nv_bfloat16>(shadow);
  a.n = p.numel();
  a.lr = ptr<float>(lr);
  a.step = ptr<float>(step);
  a.gscale = opt_ptr<float>(gscale);
  a.beta1 = (float)beta1; a.beta2 = (float)beta2; a.eps = (float)eps; a.wd = (float)wd;
  a.decoupled = decoupled;
  a.zero_grad = zero_grad;
  c10::cuda::CUDAGuard guard(p.device());
  FL_CUDA_OK(flodl::launch_adamw(a, cur_stream()));
}

void sgd(Tensor& p, Tensor& g, const optional<Tensor>& buf, const optional<Tensor>& shadow,
         const Tensor& lr, const optional<Tensor>& gscale, const optional<Tensor>& first,
         double momentum, double dampening, double wd, bool nesterov, bool zero_grad) {
  FL_CHECK_F32(p); FL_CHECK_F32(g);
  flodl::SgdArgs a;
  a.p = ptr<float>(p); a.g = ptr<float>(g);
  a.buf = opt_ptr<float>(buf);
  a.shadow = opt_ptr<__nv_bfloat16>(shadow);
  a.n = p.numel();
  a.lr = ptr<float>(lr);
  a.gscale = opt_ptr<float>(gscale);
  a.first = opt_ptr<float>(first);
  a.momentum = (float)momentum; a.dampening = (float)dampening; a.wd = (float)wd;
  a.nesterov = nesterov;
  a.zero_grad = zero_grad;
  c10::cuda::CUDAGuard guard(p.device());
  FL_CUDA_OK(flodl::launch_sgd(a, cur_stream()));
}

void sumsq(const Tensor& x, Tensor& out) {
  FL_CHECK_F32(x);
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_sumsq(ptr<float>(x), x.numel(), ptr<float>(out), cur_stream()));
}

void clip_coef(const Tensor& sumsq_t, double max_norm, Tensor& coef, const optional<Tensor>& norm) {
  c10::cuda::CUDAGuard guard(coef.device());
  FL_CUDA_OK(flodl::launch_clip_coef(ptr<float>(sumsq_t), (float)max_norm, ptr<float>(coef),
                                     opt_ptr<float>(norm), cur_stream()));
}

void add_scalar(Tensor& x, double v) {
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_add_scalar(ptr<float>(x), (float)v, cur_stream()));
}

void cast_f32_bf16(const Tensor& x, Tensor& y) {
  FL_CHECK_F32(x); FL_CHECK_BF16(y);
  FL_CHECK(x.numel() == y.numel() && x.is_contiguous() && y.is_contiguous(), "cast sizes");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_cast_f32_bf16(ptr<float>(x), ptr<__nv_bfloat16>(y), x.numel(), cur_stream()));
}

void gelu_bwd(const Tensor& dy, const Tensor& h, Tensor& dh) {
  FL_CHECK_BF16(dy); FL_CHECK_BF16(h); FL_CHECK_BF16(dh);
  FL_CHECK(dy.numel() == h.numel() && dh.numel() == h.numel(), "gelu_bwd sizes");
  FL_CHECK(dy.is_contiguous() && h.is_contiguous() && dh.is_contiguous(), "gelu_bwd layout");
  c10::cuda::CUDAGuard guard(h.device());
  FL_CUDA_OK(flodl::launch_gelu_bwd(ptr<__nv_bfloat16>(dy), ptr<__nv_bfloat16>(h),
                                    ptr<__nv_bfloat16>(dh), h.numel(), cur_stream()));
}

void mul_bf16(const Tensor& a, const Tensor& b, Tensor& y) {
  FL_CHECK_CUDA(a);
  FL_CHECK_BF16(a);
  FL_CHECK_BF16(b);
  FL_CHECK_BF16(y);
  FL_CHECK(a.is_contiguous() && b.is_contiguous() && y.is_contiguous() &&
               a.numel() == b.numel() && a.numel() == y.numel(),
           "mul_bf16 layout");
  c10::cuda::CUDAGuard guard(a.device());
  FL_CUDA_OK(flodl::launch_mul_bf16(ptr<__nv_bfloat16>(a), ptr<__nv_bfloat16>(b),
                                    ptr<__nv_bfloat16>(y), a.numel(), cur_stream()));
}

void gelu_eval_f32(const Tensor& x, Tensor& y, Tensor& dydx) {
  FL_CHECK_CUDA(x);
  FL_CHECK_F32(x);
  FL_CHECK_F32(y);
  FL_CHECK_F32(dydx);
  FL_CHECK(x.is_contiguous() && y.is_contiguous() && dydx.is_contiguous() &&
               x.numel() == y.numel() && x.numel() == dydx.numel(),
           "gelu_eval_f32 layout");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_gelu_eval_f32(x.data_ptr<float>(), y.data_ptr<float>(),
                                         dydx.data_ptr<float>(), x.numel(), cur_stream()));
}

void gelu_fwd(const Tensor& x, Tensor& y) {
  FL_CHECK_BF16(x); FL_CHECK_BF16(y);
  FL_CHECK(x.is_contiguous() && y.is_contiguous() && x.numel() == y.numel(), "gelu_fwd layout");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_gelu_fwd(ptr<__nv_bfloat16>(x), ptr<__nv_bfloat16>(y), x.numel(),
                                    cur_stream()));
}

}  // namespace

void register_norm(py::module& m) {
  m.def("ln_fwd", &ln_fwd, py::arg("x"), py::arg("gamma"), py::arg("beta"), py::arg("y_bf16"),
        py::arg("y_f32"), py::arg("mean"), py::arg("rstd"), py::arg("eps"));
  m.def("ln_bwd", &ln_bwd, py::arg("dy"), py::arg("x"), py::arg("mean"), py::arg("rstd"),
        py::arg("gamma"), py::arg("dres"), py::arg("dx_f32"), py::arg("dx_bf16"),
        py::arg("dgamma"), py::arg("dbeta"), py::arg("colsum"), py::arg("pre_add") = false);
  m.def("colsum", &colsum, py::arg("m"), py::arg("out"), py::arg("scale") = py::none());
}

void register_loss(py::module& m) {
  m.def("softmax_ce", &softmax_ce, py::arg("logits"), py::arg("targets"), py::arg("loss"),
        py::arg("inv_count"), py::arg("dlogits"), py::arg("ignore_index"), py::arg("smoothing"));
}

void register_elementwise(py::module& m) {
  m.def("embed_fwd", &embed_fwd, py::arg("ids"), py::arg("tok"), py::arg("pos"),
        py::arg("type_ids"), py::arg("type_tab"), py::arg("out"), py::arg("out_bf16"), py::arg("S"));
  m.def("embed_bwd_atomic", &embed_bwd_atomic);
  m.def("pos_grad", &pos_grad);
  m.def("onehot_bf16", &onehot_bf16);
  m.def("cast_f32_bf16", &cast_f32_bf16);
  m.def("rms_fwd", &rms_fwd, py::arg("x"), py::arg("w"), py::arg("y"), py::arg("rstd"),
        py::arg("eps"));
  m.def("rms_bwd", &rms_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"),
        py::arg("dx"), py::arg("dw"));
  m.def("gn_fwd", &gn_fwd, py::arg("x"), py::arg("gamma"), py::arg("beta"), py::arg("y"),
        py::arg("mean"), py::arg("rstd"), py::arg("groups"), py::arg("eps"));
  m.def("gn_bwd", &gn_bwd, py::arg("dy"), py::arg("x"), py::arg("gamma"), py::arg("mean"),
        py::arg("rstd"), py::arg("dx"), py::arg("dgamma"), py::arg("dbeta"), py::arg("groups"));
  m.def("maxpool_fwd", &maxpool_fwd);
  m.def("maxpool_bwd", &maxpool_bwd);
  m.def("dropout", &dropout, py::arg("x"), py::arg("y"), py::arg("p"), py::arg("seed"),
        py::arg("offset"));
  m.def("gelu_bwd", &gelu_bwd);
  m.def("gelu_fwd", &gelu_fwd);
  m.def("gelu_eval_f32", &gelu_eval_f32);
  m.def("mul_bf16", &mul_bf16);
}

void register_optim(py::module& m) {
  m.def("adamw", &adamw, py::arg("p"), py::arg("g"), py::arg("m"), py::arg("v"),
        py::arg("shadow"), py::arg("lr"), py::arg("step"), py::arg("gscale"), py::arg("beta1"),
        py::arg("beta2"), py::arg("eps"), py::arg("wd"), py::arg("decoupled"),
        py::arg("zero_grad"));
  m.def("sgd", &sgd, py::arg("p"), py::arg("g"), py::arg("buf"), py::arg("shadow"), py::arg("lr"),
        py::arg("gscale"), py::arg("first"), py::arg("momentum"), py::arg("dampening"),
        py::arg("wd"), py::arg("nesterov"), py::arg("zero_grad"));
  m.def("sumsq", &sumsq);
  m.def("clip_coef", &clip_coef, py::arg("sumsq"), py::arg("max_norm"), py::arg("coef"),
        py::arg("norm") = py::none());
  m.def("add_scalar", &add_scalar);
}
