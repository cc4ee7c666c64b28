// Python module of the sm_100a kernel library (flodl_b200._C).
#include "common.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "flodl_b200 sm_100a kernel library";
  register_gemm(m);
  register_norm(m);
  register_loss(m);
  register_elementwise(m);
  register_optim(m);
  register_attention(m);
  register_comm(m);
  register_conv(m);
}
