// Python module of the native (CPU-side) runtime (flodl_b200._native).
#include "runtime.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "flodl_b200 native runtime";
  flodl::rt::register_checkpoint(m);
  flodl::rt::register_hash(m);
  flodl::rt::register_graph(m);
  flodl::rt::register_elche(m);
  flodl::rt::register_wire(m);
  flodl::rt::register_crash(m);
  flodl::rt::register_chunk_pool(m);
}
