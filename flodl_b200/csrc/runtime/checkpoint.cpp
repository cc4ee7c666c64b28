// `.fdl` checkpoint reader/writer, byte-compatible with floDl's format
// (flodl/src/nn/checkpoint.rs:9-16, 36-78, 154-200, 469-529):
//
//   "FDLC" | version u32 LE (=2) | structural hash [32] | count u32 |
//   count x { name_len u32 | name | ndim u32 | shape i64[ndim] |
//             dtype_tag u8 | byte_count u64 | raw native bytes }
//
// dtype tags: 1 f16, 2 bf16, 3 f32, 4 f64, 5 i32, 6 i64. A path ending in
// ".gz" is gzip-compressed. Writes go to "<path>.tmp" and are renamed over the
// final path, so a crash never leaves a torn checkpoint.
#include "runtime.h"

#include <zlib.h>

#include <cstdio>
#include <memory>
#include <stdexcept>

namespace flodl {
namespace rt {

namespace {

constexpr uint32_t kVersion = 2;
constexpr uint32_t kMaxVersion = 2;

uint8_t dtype_tag(at::ScalarType t) {
  switch (t) {
    case at::kHalf: return 1;
    case at::kBFloat16: return 2;
    case at::kFloat: return 3;
    case at::kDouble: return 4;
    case at::kInt: return 5;
    case at::kLong: return 6;
    default: throw std::runtime_error("checkpoint: unsupported dtype");
  }
}

at::ScalarType dtype_from_tag(uint8_t tag) {
  switch (tag) {
    case 1: return at::kHalf;
    case 2: return at::kBFloat16;
    case 3: return at::kFloat;
    case 4: return at::kDouble;
    case 5: return at::kInt;
    case 6: return at::kLong;
    default: throw std::runtime_error("unknown dtype tag: " + std::to_string(tag));
  }
}

bool ends_with(const std::string& s, const std::string& suf) {
  return s.size() >= suf.size() && s.compare(s.size() - suf.size(), suf.size(), suf) == 0;
}

// Minimal byte sink/source over either stdio or zlib.
class Writer {
 public:
  explicit Writer(const std::string& path, bool gz) : gz_(gz) {
    if (gz_) {
      g_ = gzopen(path.c_str(), "wb");
      if (!g_) throw std::runtime_error("cannot open " + path);
    } else {
      f_ = std::fopen(path.c_str(), "wb");
      if (!f_) throw std::runtime_error("cannot open " + path);
      std::setvbuf(f_, nullptr, _IOFBF, 1 << 20);
    }
  }
  ~Writer() { close(); }
  void write(const void* p, size_t n) {
    const char* c = static_cast<const char*>(p);
    while (n > 0) {
      size_t chunk = std::min<size_t>(n, 1u << 30);
      if (gz_) {
        if (gzwrite(g_, c, (unsigned)chunk) != (int)chunk)
          throw std::runtime_error("checkpoint: gzip write failed");
      } else if (std::fwrite(c, 1, chunk, f_) != chunk) {
        throw std::runtime_error("checkpoint: write failed");
      }
      c += chunk;
      n -= chunk;
    }
  }
  void u32(uint32_t v) { write(&v, 4); }  // host is little-endian (x86-64 / aarch64)
  void u64(uint64_t v) { write(&v, 8); }
  void close() {
    if (gz_ && g_) {
      if (gzclose(g_) != Z_OK) throw std::runtime_error("checkpoint: gzip close failed");
      g_ = nullptr;
    }
    if (!gz_ && f_) {
      if (std::fclose(f_) != 0) throw std::runtime_error("checkpoint: close failed");
      f_ = nullptr;
    }
  }

 private:
  bool gz_;
  gzFile g_ = nullptr;
  FILE* f_ = nullptr;
};

class Reader {
 public:
  explicit Reader(const std::string& path) : gz_(ends_with(path, ".gz")) {
    if (gz_) {
      g_ = gzopen(path.c_str(), "rb");
      if (!g_) throw std::runtime_error("cannot open " + path);
    } else {
      f_ = std::fopen(path.c_str(), "rb");
      if (!f_) throw std::runtime_error("cannot open " + path);
    }
  }
  ~Reader() {
    if (g_) gzclose(g_);
    if (f_) std::fclose(f_);
  }
  void read(void* p, size_t n) {
    char* c = static_cast<char*>(p);
    while (n > 0) {
      size_t chunk = std::min<size_t>(n, 1u << 30);
      size_t got = gz_ ? (size_t)std::max(0, gzread(g_, c, (unsigned)chunk))
                       : std::fread(c, 1, chunk, f_);
      if (got != chunk) throw std::runtime_error("checkpoint: unexpected end of file");
      c += chunk;
      n -= chunk;
    }
  }
  void skip(uint64_t n) {
    char buf[1 << 16];
    while (n > 0) {
      size_t chunk = std::min<uint64_t>(n, sizeof(buf));
      read(buf, chunk);
      n -= chunk;
    }
  }
  uint32_t u32() { uint32_t v; read(&v, 4); return v; }
  uint64_t u64() { uint64_t v; read(&v, 8); return v; }

 private:
  bool gz_;
  gzFile g_ = nullptr;
  FILE* f_ = nullptr;
};

std::array<uint8_t, 32> parse_hash(const c10::optional<std::string>& hex) {
  std::array<uint8_t, 32> h{};
  if (!hex || hex->empty()) return h;
  if (hex->size() != 64) throw std::runtime_error("structural hash must be 64 hex chars");
  for (int i = 0; i < 32; ++i) h[i] = (uint8_t)std::stoul(hex->substr(2 * i, 2), nullptr, 16);
  return h;
}

struct Header {
  uint32_t version;
  std::array<uint8_t, 32> hash;
  uint32_t count;
};

Header read_header(Reader& r) {
  char magic[4];
  r.read(magic, 4);
  if (std::string(magic, 4) != "FDLC")
    throw std::runtime_error("invalid checkpoint: bad magic (expected .fdl checkpoint)");
  Header h;
  h.version = r.u32();
  if (h.version == 0 || h.version > kMaxVersion)
    throw std::runtime_error("unsupported checkpoint version " + std::to_string(h.version) +
                             " (this build supports 1..=2)");
  r.read(h.hash.data(), 32);
  h.count = r.u32();
  return h;
}

std::string read_name(Reader& r) {
  uint32_t n = r.u32();
  if (n > (1u << 20)) throw std::runtime_error("checkpoint: entry name too long");
  std::string s(n, '\0');
  r.read(&s[0], n);
  return s;
}

std::vector<int64_t> read_shape(Reader& r) {
  uint32_t nd = r.u32();
  if (nd > 64) throw std::runtime_error("checkpoint: too many dims");
  std::vector<int64_t> shape(nd);
  for (auto& d : shape) d = (int64_t)r.u64();
  return shape;
}

void write_tensor_body(Writer& w, const at::Tensor& t_in) {
  at::Tensor t = t_in.detach().to(at::kCPU).contiguous();
  w.u32((uint32_t)t.dim());
  for (int64_t d : t.sizes()) w.u64((uint64_t)d);
  uint8_t tag = dtype_tag(t.scalar_type());
  w.write(&tag, 1);
  uint64_t bytes = (uint64_t)t.numel() * t.element_size();
  w.u64(bytes);
  if (bytes) w.write(t.data_ptr(), bytes);
}

at::Tensor read_tensor_body(Reader& r) {
  auto shape = read_shape(r);
  uint8_t tag;
  r.read(&tag, 1);
  auto dt = dtype_from_tag(tag);
  uint64_t bytes = r.u64();
  at::Tensor t = at::empty(shape, at::TensorOptions().dtype(dt));
  if ((uint64_t)t.numel() * t.element_size() != bytes)
    throw std::runtime_error("checkpoint: byte count does not match shape");
  if (bytes) r.read(t.data_ptr(), bytes);
  return t;
}

// entries: list of (name, tensor)
void write_fdl(const std::string& path, const std::vector<std::pair<std::string, at::Tensor>>& entries,
               const c10::optional<std::string>& hash_hex) {
  auto hash = parse_hash(hash_hex);
  const std::string tmp = path + ".tmp";
  try {
    Writer w(tmp, ends_with(path, ".gz"));
    w.write("FDLC", 4);
    w.u32(kVersion);
    w.write(hash.data(), 32);
    w.u32((uint32_t)entries.size());
    for (const auto& e : entries) {
      w.u32((uint32_t)e.first.size());
      w.write(e.first.data(), e.first.size());
      write_tensor_body(w, e.second);
    }
    w.close();
  } catch (...) {
    std::remove(tmp.c_str());
    throw;
  }
  if (std::rename(tmp.c_str(), path.c_str()) != 0)
    throw std::runtime_error("checkpoint: rename failed for " + path);
}

py::tuple read_fdl(const std::string& path) {
  Reader r(path);
  Header h = read_header(r);
  py::list entries;
  for (uint32_t i = 0; i < h.count; ++i) {
    std::string name = read_name(r);
    at::Tensor t = read_tensor_body(r);
    entries.append(py::make_tuple(name, t));
  }
  return py::make_tuple(h.version, to_hex(h.hash.data(), 32), entries);
}

std::vector<std::string> fdl_keys(const std::string& path) {
  Reader r(path);
  Header h = read_header(r);
  std::vector<std::string> keys;
  for (uint32_t i = 0; i < h.count; ++i) {
    keys.push_back(read_name(r));
    read_shape(r);
    uint8_t tag;
    r.read(&tag, 1);
    r.skip(r.u64());
  }
  return keys;
}

uint32_t fdl_version(const std::string& path) {
  Reader r(path);
  char magic[4];
  r.read(magic, 4);
  if (std::string(magic, 4) != "FDLC")
    throw std::runtime_error("invalid checkpoint: bad magic (expected .fdl checkpoint)");
  return r.u32();
}

// Optional-tensor state stream used by optimizer `.optim` files: a presence
// byte followed by a tensor body (flodl/src/nn/checkpoint.rs write_tensor_state).
py::bytes encode_tensor_state(const c10::optional<at::Tensor>& t) {
  // Encode into a memory buffer via a temporary file-free path.
  std::string out;
  auto put = [&](const void* p, size_t n) { out.append(static_cast<const char*>(p), n); };
  uint8_t present = t.has_value() && t->defined() ? 1 : 0;
  put(&present, 1);
  if (present) {
    at::Tensor c = t->detach().to(at::kCPU).contiguous();
    uint32_t nd = (uint32_t)c.dim();
    put(&nd, 4);
    for (int64_t d : c.sizes()) put(&d, 8);
    uint8_t tag = dtype_tag(c.scalar_type());
    put(&tag, 1);
    uint64_t bytes = (uint64_t)c.numel() * c.element_size();
    put(&bytes, 8);
    put(c.data_ptr(), bytes);
  }
  return py::bytes(out);
}

}  // namespace

void register_checkpoint(py::module& m) {
  m.def("write_fdl", &write_fdl, py::arg("path"), py::arg("entries"),
        py::arg("structural_hash") = py::none(),
        py::call_guard<py::gil_scoped_release>());
  m.def("read_fdl", &read_fdl, py::arg("path"));
  m.def("fdl_keys", &fdl_keys, py::arg("path"));
  m.def("fdl_version", &fdl_version, py::arg("path"));
  m.def("encode_tensor_state", &encode_tensor_state);
}

}  // namespace rt
}  // namespace flodl
