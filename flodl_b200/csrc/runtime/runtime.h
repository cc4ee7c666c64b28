// Native CPU runtime of flodl_b200: shared declarations.
#pragma once
#include <torch/extension.h>

#include <cstdint>
#include <string>
#include <vector>

namespace flodl {
namespace rt {

namespace py = pybind11;

// SHA-256 (FIPS 180-4) with an incremental interface.
class Sha256 {
 public:
  Sha256();
  void update(const void* data, size_t len);
  void update(const std::string& s) { update(s.data(), s.size()); }
  std::array<uint8_t, 32> digest();  // finalises; object must not be reused
  std::string hexdigest();

 private:
  void block(const uint8_t* p);
  uint32_t h_[8];
  uint8_t buf_[64];
  size_t buf_len_ = 0;
  uint64_t total_ = 0;
};

std::array<uint8_t, 32> hmac_sha256(const std::string& key, const std::string& msg);
std::string to_hex(const uint8_t* p, size_t n);

void register_checkpoint(py::module& m);
void register_hash(py::module& m);
void register_graph(py::module& m);
void register_elche(py::module& m);
void register_reduce(py::module& m);
void register_loader(py::module& m);
void register_wire(py::module& m);
void register_crash(py::module& m);
void register_chunk_pool(py::module& m);
void install_crash_handler();

}  // namespace rt
}  // namespace flodl
