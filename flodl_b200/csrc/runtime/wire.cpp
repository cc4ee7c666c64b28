// Signed wire frames and the CPU averaging reducer (native).
//
// Frames carry control, rendezvous, timing and CPU-averaging payloads between
// ranks, relays and the controller (reference roles: flodl/src/distributed/
// wire.rs:79-154, 488-568, 826-960). Layout, little-endian:
//
//   magic u32 | version u8 | kind u8 | flags u16 | seq u64 | len u64 |
//   payload[len] | tag u64
//
// tag = first 8 bytes of HMAC-SHA256(key, header || payload). Frames above
// `max_len` are rejected before any allocation; tags are compared in constant
// time.
//
// CPU reduce (controller/round_frame.rs:517-540 semantics): payloads arrive
// pre-scaled by their mass; the reducer sums payloads and masses and divides
// once by the accepted mass. Summation runs multi-threaded over chunks.
#include "runtime.h"

#include <cstring>
#include <stdexcept>
#include <thread>

namespace flodl {
namespace rt {

namespace {

constexpr uint8_t kWireVersion = 1;
constexpr size_t kHeader = 4 + 1 + 1 + 2 + 8 + 8;

template <typename T>
void put(std::string& s, T v) {
  s.append(reinterpret_cast<const char*>(&v), sizeof(T));
}
template <typename T>
T get(const char* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));
  return v;
}

uint64_t tag64(const std::string& key, const std::string& body) {
  auto d = hmac_sha256(key, body);
  uint64_t t;
  std::memcpy(&t, d.data(), 8);
  return t;
}

py::bytes encode_frame(uint32_t magic, int kind, uint64_t seq, py::bytes payload_b,
                       py::bytes key_b, int flags) {
  std::string payload = payload_b, key = key_b;
  std::string out;
  out.reserve(kHeader + payload.size() + 8);
  put<uint32_t>(out, magic);
  put<uint8_t>(out, kWireVersion);
  put<uint8_t>(out, (uint8_t)kind);
  put<uint16_t>(out, (uint16_t)flags);
  put<uint64_t>(out, seq);
  put<uint64_t>(out, (uint64_t)payload.size());
  out += payload;
  put<uint64_t>(out, tag64(key, out));
  return py::bytes(out);
}

// Returns (magic, kind, flags, seq, payload). Raises on bad version, length,
// or signature.
py::tuple decode_frame(py::bytes frame_b, py::bytes key_b, uint64_t max_len) {
  std::string f = frame_b, key = key_b;
  if (f.size() < kHeader + 8) throw std::runtime_error("wire: frame too short");
  const char* p = f.data();
  const uint32_t magic = get<uint32_t>(p);
  const uint8_t ver = get<uint8_t>(p + 4);
  const uint8_t kind = get<uint8_t>(p + 5);
  const uint16_t flags = get<uint16_t>(p + 6);
  const uint64_t seq = get<uint64_t>(p + 8);
  const uint64_t len = get<uint64_t>(p + 16);
  if (ver != kWireVersion) throw std::runtime_error("wire: unsupported frame version");
  if (len > max_len) throw std::runtime_error("wire: frame exceeds the size ceiling");
  if (f.size() != kHeader + len + 8) throw std::runtime_error("wire: length mismatch");
  const uint64_t want = tag64(key, f.substr(0, kHeader + len));
  const uint64_t got = get<uint64_t>(p + kHeader + len);
  uint64_t diff = want ^ got;  // constant-time compare
  if (diff != 0) throw std::runtime_error("wire: bad signature");
  return py::make_tuple(magic, (int)kind, (int)flags, seq, py::bytes(f.substr(kHeader, len)));
}

// Parse just the header of a frame prefix: (magic, kind, flags, seq, len) so a
// reader knows how many more bytes to receive.
py::tuple peek_header(py::bytes hdr_b) {
  std::string h = hdr_b;
  if (h.size() < kHeader) throw std::runtime_error("wire: short header");
  const char* p = h.data();
  return py::make_tuple(get<uint32_t>(p), (int)get<uint8_t>(p + 5), (int)get<uint16_t>(p + 6),
                        get<uint64_t>(p + 8), get<uint64_t>(p + 16));
}

// out = sum_i payload_i ; mass = sum_i mass_i ; out /= mass (once).
at::Tensor reduce_scaled(const std::vector<at::Tensor>& payloads, const std::vector<double>& masses,
                         int threads) {
  if (payloads.empty()) throw std::runtime_error("reduce: no payloads");
  if (payloads.size() != masses.size()) throw std::runtime_error("reduce: mass per payload");
  const int64_t n = payloads[0].numel();
  std::vector<const float*> src;
  for (const auto& t : payloads) {
    if (t.scalar_type() != at::kFloat || !t.is_contiguous() || t.device().type() != at::kCPU ||
        t.numel() != n)
      throw std::runtime_error("reduce: payloads must be contiguous f32 CPU tensors of one size");
    src.push_back(t.data_ptr<float>());
  }
  double mass = 0.0;
  for (double m : masses) mass += m;
  at::Tensor out = at::empty({n}, at::TensorOptions().dtype(at::kFloat));
  float* o = out.data_ptr<float>();
  const float inv = mass > 0.0 ? (float)(1.0 / mass) : 0.f;
  const int T = std::max(1, std::min(threads, (int)std::max<int64_t>(1, n / (1 << 16))));
  auto work = [&](int64_t a, int64_t b) {
    for (int64_t i = a; i < b; ++i) {
      float s = 0.f;
      for (const float* p : src) s += p[i];
      o[i] = s * inv;
    }
  };
  std::vector<std::thread> pool;
  const int64_t chunk = (n + T - 1) / T;
  for (int t = 0; t < T; ++t) {
    const int64_t a = t * chunk, b = std::min(n, a + chunk);
    if (a < b) pool.emplace_back(work, a, b);
  }
  for (auto& th : pool) th.join();
  return out;
}

// bf16 wire encoding (round to nearest even) and decoding.
at::Tensor f32_to_bf16_bits(const at::Tensor& x) {
  at::Tensor c = x.contiguous();
  const float* s = c.data_ptr<float>();
  at::Tensor out = at::empty({c.numel()}, at::TensorOptions().dtype(at::kShort));
  int16_t* o = out.data_ptr<int16_t>();
  for (int64_t i = 0; i < c.numel(); ++i) {
    uint32_t u;
    std::memcpy(&u, &s[i], 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) {
      o[i] = (int16_t)((u >> 16) | 0x40);  // quiet NaN
    } else {
      const uint32_t bias = 0x7fffu + ((u >> 16) & 1u);
      o[i] = (int16_t)((u + bias) >> 16);
    }
  }
  return out;
}

at::Tensor bf16_bits_to_f32(const at::Tensor& b) {
  at::Tensor c = b.contiguous();
  const int16_t* s = c.data_ptr<int16_t>();
  at::Tensor out = at::empty({c.numel()}, at::TensorOptions().dtype(at::kFloat));
  float* o = out.data_ptr<float>();
  for (int64_t i = 0; i < c.numel(); ++i) {
    const uint32_t u = ((uint32_t)(uint16_t)s[i]) << 16;
    std::memcpy(&o[i], &u, 4);
  }
  return out;
}

}  // namespace

void register_wire(py::module& m) {
  m.def("encode_frame", &encode_frame, py::arg("magic"), py::arg("kind"), py::arg("seq"),
        py::arg("payload"), py::arg("key"), py::arg("flags") = 0);
  m.def("decode_frame", &decode_frame, py::arg("frame"), py::arg("key"),
        py::arg("max_len") = (uint64_t)1 << 34);
  m.def("peek_header", &peek_header);
  m.attr("WIRE_HEADER_BYTES") = (int)kHeader;
  m.def("reduce_scaled", &reduce_scaled, py::arg("payloads"), py::arg("masses"),
        py::arg("threads") = 8, py::call_guard<py::gil_scoped_release>());
  m.def("f32_to_bf16_bits", &f32_to_bf16_bits);
  m.def("bf16_bits_to_f32", &bf16_bits_to_f32);
}

}  // namespace rt
}  // namespace flodl
