// Torch bindings of the peer-memory communicator: symmetric allocation with
// CUDA IPC handles, peer mapping, host-mapped error words and the fused
// collective launches.
#include "common.h"
#include "../comm/peer_comm.h"

#include <cstring>
#include <string>
#include <vector>

namespace {

using at::Tensor;

// cudaMalloc a region and return (device pointer, IPC handle bytes).
py::tuple peer_alloc(int64_t nbytes) {
  void* p = nullptr;
  FL_CUDA_OK(cudaMalloc(&p, (size_t)nbytes));
  FL_CUDA_OK(cudaMemset(p, 0, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  FL_CUDA_OK(cudaIpcGetMemHandle(&h, p));
  return py::make_tuple(reinterpret_cast<int64_t>(p),
                        py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

int64_t peer_open(py::bytes handle) {
  std::string s = handle;
  FL_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  FL_CUDA_OK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void peer_close(int64_t ptr) { FL_CUDA_OK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

void peer_free(int64_t ptr) { FL_CUDA_OK(cudaFree(reinterpret_cast<void*>(ptr))); }

// Non-owning tensor view of device memory allocated above.
Tensor tensor_from_ptr(int64_t ptr, int64_t numel, const std::string& dtype, int64_t device) {
  at::ScalarType st;
  if (dtype == "float32") st = at::kFloat;
  else if (dtype == "bfloat16") st = at::kBFloat16;
  else if (dtype == "int32") st = at::kInt;
  else TORCH_CHECK(false, "tensor_from_ptr: unsupported dtype ", dtype);
  auto opts = at::TensorOptions().dtype(st).device(at::Device(at::kCUDA, (int)device));
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {}, opts);
}

// Host-mapped pinned words: returns (cpu tensor view, device pointer).
py::tuple host_mapped_words(int64_t n) {
  void* hp = nullptr;
  FL_CUDA_OK(cudaHostAlloc(&hp, (size_t)n * 4, cudaHostAllocMapped));
  std::memset(hp, 0, (size_t)n * 4);
  void* dp = nullptr;
  FL_CUDA_OK(cudaHostGetDevicePointer(&dp, hp, 0));
  Tensor t = torch::from_blob(hp, {n}, [](void* p) { cudaFreeHost(p); },
                              at::TensorOptions().dtype(at::kInt));
  return py::make_tuple(t, reinterpret_cast<int64_t>(dp));
}

void fused_launch(int64_t op, py::dict cfg, const std::vector<int64_t>& data,
                  const std::vector<int64_t>& grad, const std::vector<int64_t>& shadow,
                  const std::vector<int64_t>& sig) {
  flodl::FusedArgs a;
  auto geti = [&](const char* k, int64_t d) {
    return cfg.contains(k) ? cfg[k].cast<int64_t>() : d;
  };
  auto getf = [&](const char* k, double d) {
    return cfg.contains(k) ? cfg[k].cast<double>() : d;
  };
  auto getp = [&](const char* k) -> int64_t {
    if (!cfg.contains(k) || cfg[k].is_none()) return 0;
    py::object o = cfg[k];
    if (py::isinstance<py::int_>(o)) return o.cast<int64_t>();
    return reinterpret_cast<int64_t>(o.cast<Tensor>().data_ptr());
  };
  a.rank = (int)geti("rank", 0);
  a.world = (int)geti("world", 1);
  a.root = (int)geti("root", 0);
  a.bucket = (int)geti("bucket", 0);
  a.start = geti("start", 0);
  a.end = geti("end", 0);
  a.blocks = (int)geti("blocks", 0);
  a.threads = (int)geti("threads", 512);
  a.oneshot = geti("oneshot", 0) != 0;
  FL_CHECK(a.threads == 128 || a.threads == 256 || a.threads == 512, "threads must be 128, 256 or 512");
  FL_CHECK(a.bucket >= 0 && a.bucket < flodl::kMaxSlots, "signal slot out of range");
  a.m = reinterpret_cast<float*>(getp("m"));
  a.v = reinterpret_cast<float*>(getp("v"));
  a.lr = reinterpret_cast<const float*>(getp("lr"));
  a.step = reinterpret_cast<const float*>(getp("step"));
  a.gscale = reinterpret_cast<const float*>(getp("gscale"));
  a.first = reinterpret_cast<const float*>(getp("first"));
  a.beta1 = (float)getf("beta1", 0.9);
  a.beta2 = (float)getf("beta2", 0.999);
  a.eps = (float)getf("eps", 1e-8);
  a.wd = (float)getf("wd", 0.0);
  a.momentum = (float)getf("momentum", 0.0);
  a.dampening = (float)getf("dampening", 0.0);
  a.nesterov = geti("nesterov", 0) != 0;
  a.average = geti("average", 1) != 0;
  a.mass = (float)getf("mass", 1.0);
  a.mover = (float)getf("mover", 1.0);
  a.buf_start = geti("buf_start", -1);
  a.div = reinterpret_cast<float*>(getp("div"));
  a.sumsq = reinterpret_cast<float*>(getp("sumsq"));
  a.norm_out = reinterpret_cast<float*>(getp("norm_out"));
  a.max_norm = (float)getf("max_norm", 0.0);
  a.table = reinterpret_cast<const int64_t*>(getp("table"));
  a.nb = (int)geti("nb", 0);
  a.timeout_ns = (uint64_t)geti("timeout_ns", 10000000000LL);
  a.err = reinterpret_cast<uint32_t*>(getp("err"));
  FL_CHECK(a.world >= 1 && a.world <= flodl::kMaxRanks, "world size out of range");
  FL_CHECK(a.rank >= 0 && a.rank < a.world, "rank out of range");
  FL_CHECK((int)data.size() == a.world && (int)grad.size() == a.world &&
               (int)shadow.size() == a.world && (int)sig.size() == a.world,
           "one pointer per rank required");
  if (op == (int64_t)flodl::FusedOp::kArAdamW || op == (int64_t)flodl::FusedOp::kClipApplyAdamW)
    FL_CHECK(a.m && a.v && a.lr && a.step, "fused AdamW needs m, v, lr, step");
  if (op == (int64_t)flodl::FusedOp::kArSgd || op == (int64_t)flodl::FusedOp::kClipApplySgd)
    FL_CHECK(a.lr, "fused SGD needs lr");
  if (op == (int64_t)flodl::FusedOp::kReduceScatter || op == (int64_t)flodl::FusedOp::kClipApplyAdamW ||
      op == (int64_t)flodl::FusedOp::kClipApplySgd)
    FL_CHECK(a.sumsq, "clip mode needs the sum-of-squares accumulator");
  if (op == (int64_t)flodl::FusedOp::kClipApplyAdamW || op == (int64_t)flodl::FusedOp::kClipApplySgd)
    FL_CHECK(a.table && a.nb > 0, "clip apply needs the bucket table");
  flodl::PeerPtrs ptrs;
  for (int p = 0; p < flodl::kMaxRanks; ++p) {
    ptrs.data[p] = p < a.world ? reinterpret_cast<float*>(data[p]) : nullptr;
    ptrs.grad[p] = p < a.world ? reinterpret_cast<float*>(grad[p]) : nullptr;
    ptrs.shadow[p] = p < a.world ? reinterpret_cast<__nv_bfloat16*>(shadow[p]) : nullptr;
    ptrs.sig[p] = p < a.world ? reinterpret_cast<uint32_t*>(sig[p]) : nullptr;
  }
  FL_CUDA_OK(flodl::launch_fused(static_cast<flodl::FusedOp>(op), a, ptrs, cur_stream()));
}

}  // namespace

void register_comm(py::module& m) {
  m.def("peer_alloc", &peer_alloc);
  m.def("peer_open", &peer_open);
  m.def("peer_close", &peer_close);
  m.def("peer_free", &peer_free);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("host_mapped_words", &host_mapped_words);
  m.def("fused_launch", &fused_launch);
  m.def("signal_words", &flodl::signal_words);
  m.attr("FUSED_AR_ADAMW") = (int)flodl::FusedOp::kArAdamW;
  m.attr("FUSED_AR_SGD") = (int)flodl::FusedOp::kArSgd;
  m.attr("FUSED_ALL_REDUCE") = (int)flodl::FusedOp::kAllReduce;
  m.attr("FUSED_WEIGHTED_AVG") = (int)flodl::FusedOp::kWeightedAverage;
  m.attr("FUSED_BROADCAST") = (int)flodl::FusedOp::kBroadcast;
  m.attr("FUSED_REDUCE_SCATTER") = (int)flodl::FusedOp::kReduceScatter;
  m.attr("FUSED_CLIP_APPLY_ADAMW") = (int)flodl::FusedOp::kClipApplyAdamW;
  m.attr("FUSED_CLIP_APPLY_SGD") = (int)flodl::FusedOp::kClipApplySgd;
  m.attr("MAX_RANKS") = flodl::kMaxRanks;
  m.attr("MAX_BUCKETS") = flodl::kMaxBuckets;
  m.attr("MAX_SLOTS") = flodl::kMaxSlots;
  m.attr("MAX_BLOCKS") = flodl::kMaxBlocks;
}
