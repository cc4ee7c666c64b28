// Torch bindings of the convolution / batch-norm building blocks (conv.cu).
#include "common.h"
#include "../kernels/kernels.h"

namespace {

using at::Tensor;
using c10::optional;

template <typename T>
T* ptr(const Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}

void check_nhwc(const Tensor& x, const char* what) {
  FL_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 4 && x.is_contiguous(),
           what, " must be a contiguous NHWC bf16 CUDA tensor [N, H, W, C]");
}

// cols [N*Ho*Wo, k*k*C] bf16, column (kh*k + kw)*C + ci (C a multiple of 8)
void im2col(const Tensor& x, Tensor& cols, int64_t k, int64_t s, int64_t p) {
  check_nhwc(x, "x");
  FL_CHECK(cols.scalar_type() == at::kBFloat16 && cols.dim() == 2 && cols.is_contiguous(),
           "cols must be contiguous bf16 [M, k*k*C]");
  const int N = (int)x.size(0), H = (int)x.size(1), W = (int)x.size(2), C = (int)x.size(3);
  FL_CHECK(C % 8 == 0, "im2col needs a multiple of 8 channels");
  const int Ho = (H + 2 * (int)p - (int)k) / (int)s + 1, Wo = (W + 2 * (int)p - (int)k) / (int)s + 1;
  FL_CHECK(cols.size(0) == (int64_t)N * Ho * Wo && cols.size(1) == C * k * k, "cols shape");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_im2col(ptr<__nv_bfloat16>(x), ptr<__nv_bfloat16>(cols), N, H, W, C,
                                  (int)k, (int)s, (int)p, cur_stream()));
}

// dx [N, H, W, C] = col2im(dcols) (+ add) (* [mask > 0])
void col2im(const Tensor& dcols, Tensor& dx, int64_t k, int64_t s, int64_t p,
            const optional<Tensor>& add, const optional<Tensor>& mask) {
  check_nhwc(dx, "dx");
  FL_CHECK(dcols.scalar_type() == at::kBFloat16 && dcols.dim() == 2 && dcols.stride(1) == 1,
           "dcols must be row-major bf16 [M, >= C*k*k]");
  const int N = (int)dx.size(0), H = (int)dx.size(1), W = (int)dx.size(2), C = (int)dx.size(3);
  if (add) FL_CHECK(add->is_contiguous() && add->numel() == dx.numel(), "add shape");
  if (mask) FL_CHECK(mask->is_contiguous() && mask->numel() == dx.numel() &&
                         mask->scalar_type() == at::kBFloat16, "mask must be bf16 like dx");
  c10::cuda::CUDAGuard guard(dx.device());
  FL_CUDA_OK(flodl::launch_col2im(ptr<__nv_bfloat16>(dcols), (int)dcols.stride(0),
                                  ptr<__nv_bfloat16>(dx), add ? add->data_ptr() : nullptr,
                                  add && add->scalar_type() == at::kFloat, opt_ptr<__nv_bfloat16>(mask),
                                  N, H, W, C, (int)k, (int)s, (int)p, cur_stream()));
}

// col2im whose output dx (after add and mask) is the gradient dz of a batch
// norm with input x: the same pass adds sum dz and sum dz * xhat into ws (2C+1
// f32, zeroed), and its last block writes them to sums, accumulates dgamma /
// dbeta and re-zeroes ws. bn_bwd_apply then finishes that batch norm.
void col2im_bn(const Tensor& dcols, Tensor& dx, int64_t k, int64_t s, int64_t p,
               const optional<Tensor>& add, const optional<Tensor>& mask, const Tensor& x,
               const Tensor& mean, const Tensor& rstd, const optional<Tensor>& dgamma,
               const optional<Tensor>& dbeta, Tensor& sums, Tensor& ws) {
  check_nhwc(dx, "dx");
  FL_CHECK(dcols.scalar_type() == at::kBFloat16 && dcols.dim() == 2 && dcols.stride(1) == 1,
           "dcols must be row-major bf16 [M, >= C*k*k]");
  const int N = (int)dx.size(0), H = (int)dx.size(1), W = (int)dx.size(2), C = (int)dx.size(3);
  if (add) FL_CHECK(add->is_contiguous() && add->numel() == dx.numel(), "add shape");
  if (mask) FL_CHECK(mask->is_contiguous() && mask->numel() == dx.numel() &&
                         mask->scalar_type() == at::kBFloat16, "mask must be bf16 like dx");
  FL_CHECK(x.is_contiguous() && x.scalar_type() == at::kBFloat16 && x.numel() == dx.numel(),
           "x must be bf16 like dx");
  FL_CHECK(C % 8 == 0 && 256 % (C / 8) == 0, "col2im_bn needs C / 8 to divide 256");
  FL_CHECK(mean.numel() >= C && rstd.numel() >= C && sums.numel() >= 2 * C &&
               ws.numel() >= 2 * C + 1 && ws.scalar_type() == at::kFloat,
           "col2im_bn scratch sizes");
  float* wsp = ptr<float>(ws);
  const flodl::BnBwdSums bn{ptr<__nv_bfloat16>(x), ptr<float>(mean), ptr<float>(rstd),
                            opt_ptr<float>(dgamma), opt_ptr<float>(dbeta), ptr<float>(sums), wsp,
                            reinterpret_cast<unsigned*>(wsp + 2 * C)};
  c10::cuda::CUDAGuard guard(dx.device());
  FL_CUDA_OK(flodl::launch_col2im_geo(
      ptr<__nv_bfloat16>(dcols), (int)dcols.stride(0), ptr<__nv_bfloat16>(dx),
      add ? add->data_ptr() : nullptr, add && add->scalar_type() == at::kFloat,
      opt_ptr<__nv_bfloat16>(mask), N, H, W, C,
      flodl::ConvGeo{(int)k, (int)k, (int)s, (int)s, (int)p, (int)p}, cur_stream(), &bn));
}

// Rectangular-kernel forms (per-axis kernel, stride, padding).
void im2col_geo(const Tensor& x, Tensor& cols, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                int64_t ph, int64_t pw) {
  check_nhwc(x, "x");
  FL_CHECK(cols.scalar_type() == at::kBFloat16 && cols.dim() == 2 && cols.is_contiguous(),
           "cols must be contiguous bf16 [M, kh*kw*C]");
  const int N = (int)x.size(0), H = (int)x.size(1), W = (int)x.size(2), C = (int)x.size(3);
  FL_CHECK(C % 8 == 0, "im2col needs a multiple of 8 channels");
  const int Ho = (H + 2 * (int)ph - (int)kh) / (int)sh + 1;
  const int Wo = (W + 2 * (int)pw - (int)kw) / (int)sw + 1;
  FL_CHECK(cols.size(0) == (int64_t)N * Ho * Wo && cols.size(1) == C * kh * kw, "cols shape");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_im2col_geo(ptr<__nv_bfloat16>(x), ptr<__nv_bfloat16>(cols), N, H, W, C,
                                      flodl::ConvGeo{(int)kh, (int)kw, (int)sh, (int)sw, (int)ph,
                                                     (int)pw},
                                      cur_stream()));
}

void col2im_geo(const Tensor& dcols, Tensor& dx, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                int64_t ph, int64_t pw) {
  check_nhwc(dx, "dx");
  FL_CHECK(dcols.scalar_type() == at::kBFloat16 && dcols.dim() == 2 && dcols.stride(1) == 1,
           "dcols must be row-major bf16 [M, >= C*kh*kw]");
  const int N = (int)dx.size(0), H = (int)dx.size(1), W = (int)dx.size(2), C = (int)dx.size(3);
  c10::cuda::CUDAGuard guard(dx.device());
  FL_CUDA_OK(flodl::launch_col2im_geo(ptr<__nv_bfloat16>(dcols), (int)dcols.stride(0),
                                      ptr<__nv_bfloat16>(dx), nullptr, false, nullptr, N, H, W, C,
                                      flodl::ConvGeo{(int)kh, (int)kw, (int)sh, (int)sw, (int)ph,
                                                     (int)pw},
                                      cur_stream()));
}

void bn_stats(const Tensor& x, Tensor& mean, Tensor& rstd, const optional<Tensor>& run_mean,
              const optional<Tensor>& run_var, Tensor& ws, double eps, double momentum) {
  FL_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x");
  const int C = (int)x.size(-1);
  FL_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= 2 * C + 1, "ws needs 2C+1 f32 (zeroed)");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_bn_stats(ptr<__nv_bfloat16>(x), x.numel() / C, C, (float)eps,
                                    (float)momentum, ptr<float>(mean), ptr<float>(rstd),
                                    opt_ptr<float>(run_mean), opt_ptr<float>(run_var),
                                    ptr<float>(ws), reinterpret_cast<unsigned*>(ptr<float>(ws) + 2 * C),
                                    cur_stream()));
}

// Batch norm from the statistics a convolution GEMM accumulated into ws
// (sum, sum of squares; ws[2C] is the ticket word, left zeroed).
void bn_apply_sums(const Tensor& x, Tensor& ws, Tensor& mean, Tensor& rstd,
                   const optional<Tensor>& run_mean, const optional<Tensor>& run_var,
                   const optional<Tensor>& gamma, const optional<Tensor>& beta,
                   const optional<Tensor>& identity, bool relu, Tensor& y, double eps,
                   double momentum) {
  FL_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x");
  const int C = (int)x.size(-1);
  FL_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= 2 * C + 1, "ws needs 2C+1 f32");
  FL_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.numel() == x.numel(), "y");
  if (identity) FL_CHECK(identity->scalar_type() == at::kBFloat16 && identity->is_contiguous() &&
                             identity->numel() == x.numel(), "identity");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_bn_apply_sums(
      ptr<__nv_bfloat16>(x), x.numel() / C, C, ptr<float>(ws),
      reinterpret_cast<unsigned*>(ptr<float>(ws) + 2 * C), (float)eps, (float)momentum,
      ptr<float>(mean), ptr<float>(rstd), opt_ptr<float>(run_mean), opt_ptr<float>(run_var),
      opt_ptr<const float>(gamma), opt_ptr<const float>(beta),
      opt_ptr<const __nv_bfloat16>(identity), relu, ptr<__nv_bfloat16>(y), cur_stream()));
}

void bn_apply(const Tensor& x, const Tensor& mean, const Tensor& rstd, const optional<Tensor>& gamma,
              const optional<Tensor>& beta, const optional<Tensor>& identity, bool relu, Tensor& y) {
  FL_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x");
  FL_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.numel() == x.numel(), "y");
  if (identity) FL_CHECK(identity->scalar_type() == at::kBFloat16 && identity->is_contiguous() &&
                             identity->numel() == x.numel(), "identity");
  const int C = (int)x.size(-1);
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_bn_apply(ptr<__nv_bfloat16>(x), x.numel() / C, C, ptr<float>(mean),
                                    ptr<float>(rstd), opt_ptr<const float>(gamma),
                                    opt_ptr<const float>(beta), opt_ptr<const __nv_bfloat16>(identity),
                                    relu, ptr<__nv_bfloat16>(y), cur_stream()));
}

// dx (and optionally dz = masked dy) of a training-mode batch norm; accumulates
// dgamma / dbeta. sums: 2C f32 scratch, ws: 2C+1 f32 zeroed workspace.
void bn_bwd(const Tensor& dy, const optional<Tensor>& ymask, const Tensor& x, const Tensor& mean,
            const Tensor& rstd, const optional<Tensor>& gamma, const optional<Tensor>& dgamma,
            const optional<Tensor>& dbeta, Tensor& sums, Tensor& ws, Tensor& dx,
            const optional<Tensor>& dz_out) {
  FL_CHECK(dy.scalar_type() == at::kBFloat16 && dy.is_contiguous() && x.is_contiguous() &&
               dx.is_contiguous() && dy.numel() == x.numel() && dx.numel() == x.numel(),
           "bn_bwd layouts");
  const int C = (int)x.size(-1);
  FL_CHECK(ws.numel() >= 2 * C + 1 && sums.numel() >= 2 * C, "bn_bwd scratch sizes");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_bn_bwd(
      ptr<__nv_bfloat16>(dy), opt_ptr<const __nv_bfloat16>(ymask), ptr<__nv_bfloat16>(x),
      x.numel() / C, C, ptr<float>(mean), ptr<float>(rstd), opt_ptr<const float>(gamma),
      opt_ptr<float>(dgamma), opt_ptr<float>(dbeta), ptr<float>(sums), ptr<float>(ws),
      reinterpret_cast<unsigned*>(ptr<float>(ws) + 2 * C), ptr<__nv_bfloat16>(dx),
      opt_ptr<__nv_bfloat16>(dz_out), cur_stream()));
}

// Elementwise half of bn_bwd, with sums [2C] already reduced (col2im_bn).
void bn_bwd_apply(const Tensor& dy, const optional<Tensor>& ymask, const Tensor& x,
                  const Tensor& mean, const Tensor& rstd, const optional<Tensor>& gamma,
                  const Tensor& sums, Tensor& dx, const optional<Tensor>& dz_out) {
  FL_CHECK(dy.scalar_type() == at::kBFloat16 && dy.is_contiguous() && x.is_contiguous() &&
               dx.is_contiguous() && dy.numel() == x.numel() && dx.numel() == x.numel(),
           "bn_bwd_apply layouts");
  const int C = (int)x.size(-1);
  FL_CHECK(sums.numel() >= 2 * C, "bn_bwd_apply sums size");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_bn_bwd_apply(
      ptr<__nv_bfloat16>(dy), opt_ptr<const __nv_bfloat16>(ymask), ptr<__nv_bfloat16>(x),
      x.numel() / C, C, ptr<float>(mean), ptr<float>(rstd), opt_ptr<const float>(gamma),
      ptr<float>(sums), ptr<__nv_bfloat16>(dx), opt_ptr<__nv_bfloat16>(dz_out), cur_stream()));
}

void avgpool_fwd(const Tensor& x, Tensor& y) {
  check_nhwc(x, "x");
  const int N = (int)x.size(0), HW = (int)(x.size(1) * x.size(2)), C = (int)x.size(3);
  FL_CHECK(y.scalar_type() == at::kBFloat16 && y.numel() == (int64_t)N * C && y.is_contiguous(), "y");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_avgpool_fwd(ptr<__nv_bfloat16>(x), ptr<__nv_bfloat16>(y), N, HW, C,
                                       cur_stream()));
}

void avgpool_bwd(const Tensor& dy, Tensor& dx) {
  check_nhwc(dx, "dx");
  const int N = (int)dx.size(0), HW = (int)(dx.size(1) * dx.size(2)), C = (int)dx.size(3);
  FL_CHECK(dy.scalar_type() == at::kBFloat16 && dy.dim() == 2 && dy.size(0) == N &&
               dy.size(1) == C && dy.stride(1) == 1, "dy [N, C]");
  c10::cuda::CUDAGuard guard(dx.device());
  FL_CUDA_OK(flodl::launch_avgpool_bwd(ptr<__nv_bfloat16>(dy), (int)dy.stride(0),
                                       ptr<__nv_bfloat16>(dx), N, HW, C, cur_stream()));
}

// NCHW f32 -> NHWC bf16; y may have more channels than x (zero-filled)
void nchw_to_nhwc(const Tensor& x, Tensor& y) {
  FL_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.dim() == 4 && x.is_contiguous(),
           "x must be NCHW f32");
  check_nhwc(y, "y");
  FL_CHECK(y.size(0) == x.size(0) && y.size(1) == x.size(2) && y.size(2) == x.size(3) &&
               y.size(3) >= x.size(1), "nchw_to_nhwc shapes");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_nchw_to_nhwc(ptr<float>(x), ptr<__nv_bfloat16>(y), (int)x.size(0),
                                        (int)x.size(1), (int)(x.size(2) * x.size(3)),
                                        (int)y.size(3), cur_stream()));
}

// table: device uint8 tensor holding n ConvPackEntry records
void pack_conv_weights(const Tensor& table, int64_t n, int64_t max_elems) {
  FL_CHECK(table.is_cuda() && table.numel() >= n * (int64_t)sizeof(flodl::ConvPackEntry), "table");
  c10::cuda::CUDAGuard guard(table.device());
  FL_CUDA_OK(flodl::launch_pack_conv_weights(
      reinterpret_cast<const flodl::ConvPackEntry*>(table.data_ptr()), (int)n, (int)max_elems,
      cur_stream()));
}

void unpack_conv_grads(const Tensor& table, int64_t n, int64_t max_elems) {
  FL_CHECK(table.is_cuda() && table.numel() >= n * (int64_t)sizeof(flodl::ConvPackEntry), "table");
  c10::cuda::CUDAGuard guard(table.device());
  FL_CUDA_OK(flodl::launch_unpack_conv_grads(
      reinterpret_cast<const flodl::ConvPackEntry*>(table.data_ptr()), (int)n, (int)max_elems,
      cur_stream()));
}

void cast_pad(const Tensor& x, Tensor& y) {
  FL_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous(), "x f32");
  FL_CHECK(y.scalar_type() == at::kBFloat16 && y.dim() == 2 && y.is_contiguous(), "y bf16 2-D");
  const int rows = (int)y.size(0), ld = (int)y.size(1);
  const int cols = (int)(x.numel() / rows);
  FL_CHECK(cols <= ld && (int64_t)cols * rows == x.numel(), "cast_pad shapes");
  c10::cuda::CUDAGuard guard(x.device());
  FL_CUDA_OK(flodl::launch_cast_pad(ptr<float>(x), ptr<__nv_bfloat16>(y), rows, cols, ld,
                                    cur_stream()));
}

}  // namespace

void register_conv(py::module& m) {
  m.def("im2col", &im2col, py::arg("x"), py::arg("cols"), py::arg("k"), py::arg("stride"),
        py::arg("pad"));
  m.def("col2im", &col2im, py::arg("dcols"), py::arg("dx"), py::arg("k"), py::arg("stride"),
        py::arg("pad"), py::arg("add") = py::none(), py::arg("mask") = py::none());
  m.def("col2im_bn", &col2im_bn, py::arg("dcols"), py::arg("dx"), py::arg("k"),
        py::arg("stride"), py::arg("pad"), py::arg("add"), py::arg("mask"), py::arg("x"),
        py::arg("mean"), py::arg("rstd"), py::arg("dgamma"), py::arg("dbeta"), py::arg("sums"),
        py::arg("ws"));
  m.def("bn_bwd_apply", &bn_bwd_apply, py::arg("dy"), py::arg("ymask"), py::arg("x"),
        py::arg("mean"), py::arg("rstd"), py::arg("gamma"), py::arg("sums"), py::arg("dx"),
        py::arg("dz_out") = py::none());
  m.def("im2col_geo", &im2col_geo);
  m.def("col2im_geo", &col2im_geo);
  m.def("bn_apply_sums", &bn_apply_sums, py::arg("x"), py::arg("ws"), py::arg("mean"),
        py::arg("rstd"), py::arg("run_mean"), py::arg("run_var"), py::arg("gamma"),
        py::arg("beta"), py::arg("identity"), py::arg("relu"), py::arg("y"), py::arg("eps"),
        py::arg("momentum"));
  m.def("bn_stats", &bn_stats, py::arg("x"), py::arg("mean"), py::arg("rstd"),
        py::arg("run_mean"), py::arg("run_var"), py::arg("ws"), py::arg("eps"),
        py::arg("momentum"));
  m.def("bn_apply", &bn_apply, py::arg("x"), py::arg("mean"), py::arg("rstd"), py::arg("gamma"),
        py::arg("beta"), py::arg("identity"), py::arg("relu"), py::arg("y"));
  m.def("bn_bwd", &bn_bwd, py::arg("dy"), py::arg("ymask"), py::arg("x"), py::arg("mean"),
        py::arg("rstd"), py::arg("gamma"), py::arg("dgamma"), py::arg("dbeta"), py::arg("sums"),
        py::arg("ws"), py::arg("dx"), py::arg("dz_out") = py::none());
  m.def("avgpool_fwd", &avgpool_fwd);
  m.def("avgpool_bwd", &avgpool_bwd);
  m.def("nchw_to_nhwc", &nchw_to_nhwc);
  m.def("pack_conv_weights", &pack_conv_weights);
  m.def("unpack_conv_grads", &unpack_conv_grads);
  m.attr("CONV_PACK_ENTRY_BYTES") = (int)sizeof(flodl::ConvPackEntry);
  m.def("cast_pad", &cast_pad);
}
