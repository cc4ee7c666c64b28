// Torch bindings for the flash attention kernels.
#include "common.h"
#include "../kernels/flash_attn.h"

namespace {

using at::Tensor;
using c10::optional;

void flash_fwd(const Tensor& qkv, Tensor& out, Tensor& lse2, int64_t B, int64_t S, int64_t H,
               int64_t D, bool causal, double scale, const optional<Tensor>& key_pad) {
  FL_CHECK_CUDA(qkv);
  FL_CHECK_BF16(qkv);
  FL_CHECK_BF16(out);
  FL_CHECK_F32(lse2);
  FL_CHECK(qkv.is_contiguous() && out.is_contiguous() && lse2.is_contiguous(), "layout");
  FL_CHECK(qkv.numel() == B * S * 3 * H * D && out.numel() == B * S * H * D &&
               lse2.numel() == B * H * S, "flash_fwd sizes");
  FL_CHECK(D == 64, "flash attention kernels support head_dim 64");
  flodl::FlashArgs a;
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse2 = lse2.data_ptr<float>();
  if (key_pad) {
    FL_CHECK(key_pad->scalar_type() == at::kBool && key_pad->is_contiguous() &&
                 key_pad->numel() == B * S, "key_pad must be bool [B, S]");
    a.key_pad = reinterpret_cast<const uint8_t*>(key_pad->data_ptr());
  }
  a.B = (int)B; a.S = (int)S; a.H = (int)H; a.D = (int)D;
  a.causal = causal;
  a.scale = (float)scale;
  c10::cuda::CUDAGuard guard(qkv.device());
  FL_CUDA_OK(flodl::launch_flash_fwd(a, cur_stream()));
}

void flash_bwd(const Tensor& dout, const Tensor& qkv, const Tensor& out, const Tensor& lse2,
               Tensor& dqkv, int64_t B, int64_t S, int64_t H, int64_t D, bool causal,
               double scale, const optional<Tensor>& key_pad, const optional<Tensor>& dbias) {
  FL_CHECK_BF16(dout); FL_CHECK_BF16(qkv); FL_CHECK_BF16(out); FL_CHECK_BF16(dqkv);
  FL_CHECK(dout.is_contiguous() && qkv.is_contiguous() && out.is_contiguous() &&
               dqkv.is_contiguous(), "layout");
  FL_CHECK(D == 64, "flash attention kernels support head_dim 64");
  auto opts = qkv.options().dtype(at::kFloat);
  Tensor delta = at::empty({B, H, S}, opts);
  Tensor dq_acc;
  if (flodl::flash_bwd_needs_dq_acc((int)S)) dq_acc = at::empty({B * S, H * D}, opts);
  flodl::FlashArgs a;
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse2 = lse2.data_ptr<float>();
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.delta = delta.data_ptr<float>();
  a.dq_acc = dq_acc.defined() ? dq_acc.data_ptr<float>() : nullptr;
  if (key_pad) a.key_pad = reinterpret_cast<const uint8_t*>(key_pad->data_ptr());
  if (dbias) {
    FL_CHECK_F32(*dbias);
    FL_CHECK(dbias->is_contiguous() && dbias->numel() == 3 * H * D, "dbias must be f32 [3*H*D]");
    a.dbias = dbias->data_ptr<float>();
  }
  a.B = (int)B; a.S = (int)S; a.H = (int)H; a.D = (int)D;
  a.causal = causal;
  a.scale = (float)scale;
  c10::cuda::CUDAGuard guard(qkv.device());
  FL_CUDA_OK(flodl::launch_flash_bwd(a, cur_stream()));
}

}  // namespace

void register_attention(py::module& m) {
  m.def("set_flash_wait_limit_ns", [](int64_t ns) { flodl::set_flash_wait_limit_ns((uint64_t)ns); });
  m.def("flash_attn_fwd", &flash_fwd, py::arg("qkv"), py::arg("out"), py::arg("lse2"),
        py::arg("B"), py::arg("S"), py::arg("H"), py::arg("D"), py::arg("causal"),
        py::arg("scale"), py::arg("key_pad") = py::none());
  m.def("flash_attn_bwd", &flash_bwd, py::arg("dout"), py::arg("qkv"), py::arg("out"),
        py::arg("lse2"), py::arg("dqkv"), py::arg("B"), py::arg("S"), py::arg("H"), py::arg("D"),
        py::arg("causal"), py::arg("scale"), py::arg("key_pad") = py::none(),
        py::arg("dbias") = py::none());
}
