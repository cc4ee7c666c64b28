// Graph topology compiler for FlowBuilder graphs.
//
// Given node count and (from, to) edges, computes Kahn topological levels
// (nodes of one level have no dependencies among each other), the flat
// execution order, and per-node consumer counts used to free intermediate
// slots early. Iteration follows node index order so the schedule is
// deterministic across runs (reference: flodl/src/graph/graph.rs:714-760).
#include "runtime.h"

#include <set>
#include <stdexcept>

namespace flodl {
namespace rt {

namespace {

py::tuple compile_levels(int64_t n, const std::vector<std::pair<int64_t, int64_t>>& edges) {
  std::vector<std::set<int64_t>> deps(n), dependents(n);
  for (const auto& e : edges) {
    if (e.first < 0 || e.first >= n || e.second < 0 || e.second >= n)
      throw std::runtime_error("graph edge references an unknown node");
    deps[e.second].insert(e.first);
    dependents[e.first].insert(e.second);
  }
  std::vector<int64_t> indeg(n);
  for (int64_t i = 0; i < n; ++i) indeg[i] = (int64_t)deps[i].size();
  std::vector<int64_t> queue;
  for (int64_t i = 0; i < n; ++i)
    if (indeg[i] == 0) queue.push_back(i);
  std::vector<std::vector<int64_t>> levels;
  int64_t visited = 0;
  while (!queue.empty()) {
    levels.push_back(queue);
    visited += (int64_t)queue.size();
    std::vector<int64_t> next;
    for (int64_t u : queue)
      for (int64_t v : dependents[u])
        if (--indeg[v] == 0) next.push_back(v);
    queue.swap(next);
  }
  if (visited != n) throw std::runtime_error("cycle detected in graph");
  std::vector<int64_t> order;
  for (auto& l : levels) order.insert(order.end(), l.begin(), l.end());
  std::vector<int64_t> consumers(n);
  for (int64_t i = 0; i < n; ++i) consumers[i] = (int64_t)dependents[i].size();
  return py::make_tuple(levels, order, consumers);
}

}  // namespace

void register_graph(py::module& m) {
  m.def("compile_levels", &compile_levels, py::arg("n"), py::arg("edges"));
}

}  // namespace rt
}  // namespace flodl
