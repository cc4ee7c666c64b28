// Progressive epoch dispatch with per-rank reservations (native).
//
// Reference role: flodl/src/distributed/chunk_pool.rs. An epoch's permutation
// offsets [0, total) are split into contiguous per-rank spans. A rank takes
// chunks from the front of its own span (so its upcoming data is known and can
// be staged ahead); a rank whose span is empty steals from the tail of the
// span with the largest residue - the owner moves its cursor up, thieves move
// the span's end down, so they never overlap. A dead rank's dispatched but not
// completed chunks, and its unassigned span, go to a reclaim queue that is
// served first. `uncovered_ranges` (unassigned + in flight + reclaimed,
// coalesced) is the coverage a checkpoint records; `from_coverage` rebuilds a
// pool whose only work is those holes.
#include "runtime.h"

#include <algorithm>
#include <chrono>
#include <deque>
#include <optional>
#include <stdexcept>
#include <utility>

namespace flodl {
namespace rt {

namespace {

using Range = std::pair<int64_t, int64_t>;  // (offset, size)

class ChunkPool {
 public:
  ChunkPool(int64_t epoch, int64_t total, const std::vector<int64_t>& spans)
      : epoch_(epoch), total_(total), t0_(std::chrono::steady_clock::now()) {
    int64_t acc = 0;
    for (int64_t s : spans) {
      if (s < 0) throw std::invalid_argument("chunk pool: negative span");
      start_.push_back(acc);
      acc += s;
    }
    if (acc != total) throw std::invalid_argument("chunk pool: spans must cover the epoch exactly");
    cursor_ = start_;
    end_.resize(spans.size());
    for (size_t r = 0; r < spans.size(); ++r) end_[r] = start_[r] + spans[r];
    outstanding_.resize(spans.size());
    done_.assign(spans.size(), 0);
  }

  int64_t residue(int rank) const { return end_.at(rank) - cursor_.at(rank); }
  Range reservation(int rank) const { return {cursor_.at(rank), residue(rank)}; }

  int64_t remaining() const {
    int64_t n = 0;
    for (size_t r = 0; r < cursor_.size(); ++r) n += end_[r] - cursor_[r];
    for (const auto& x : reclaimed_) n += x.second;
    return n;
  }
  int64_t in_flight(int rank) const {
    int64_t n = 0;
    for (const auto& x : outstanding_.at(rank)) n += x.second;
    return n;
  }
  bool is_epoch_done() const {
    if (remaining() != 0) return false;
    for (const auto& o : outstanding_)
      if (!o.empty()) return false;
    return true;
  }

  std::optional<Range> take_chunk(int64_t size, int rank) {
    if (size <= 0) return std::nullopt;
    check_rank(rank);
    Range chunk;
    if (!reclaimed_.empty()) {  // close coverage holes first
      Range h = reclaimed_.front();
      reclaimed_.pop_front();
      const int64_t k = std::min(h.second, size);
      if (k < h.second) reclaimed_.push_front({h.first + k, h.second - k});
      chunk = {h.first, k};
    } else if (residue(rank) > 0) {  // own span, front to back
      const int64_t k = std::min(size, residue(rank));
      chunk = {cursor_[rank], k};
      cursor_[rank] += k;
    } else {  // steal the tail of the largest residue
      int donor = 0;
      for (int r = 1; r < (int)cursor_.size(); ++r)
        if (residue(r) > residue(donor)) donor = r;
      if (residue(donor) <= 0) return std::nullopt;
      const int64_t k = std::min(size, residue(donor));
      end_[donor] -= k;
      chunk = {end_[donor], k};
    }
    outstanding_[rank].push_back(chunk);
    return chunk;
  }

  void rollback_take(int rank, int64_t offset, int64_t size) {
    check_rank(rank);
    auto& out = outstanding_[rank];
    if (out.empty() || out.back() != Range{offset, size})
      throw std::invalid_argument("rollback must name the rank's newest outstanding chunk");
    out.pop_back();
    if (cursor_[rank] == offset + size && start_[rank] <= offset)
      cursor_[rank] = offset;
    else
      reclaimed_.push_front({offset, size});
  }

  void mark_completed(int rank, int64_t samples) {
    check_rank(rank);
    auto& out = outstanding_[rank];
    int64_t left = samples;
    while (left > 0 && !out.empty()) {
      Range& f = out.front();
      if (f.second <= left) {
        left -= f.second;
        out.pop_front();
      } else {
        f.first += left;
        f.second -= left;
        left = 0;
      }
    }
    const int64_t done = samples - left;  // a falsely-dead rank reporting late is clamped
    completed_ += done;
    done_[rank] += done;
  }

  int64_t forfeit(int rank) {
    check_rank(rank);
    int64_t n = 0;
    for (const auto& c : outstanding_[rank]) {
      reclaimed_.push_back(c);
      n += c.second;
    }
    outstanding_[rank].clear();
    if (residue(rank) > 0) {
      reclaimed_.push_back({cursor_[rank], residue(rank)});
      n += residue(rank);
      cursor_[rank] = end_[rank];
    }
    return n;
  }

  std::vector<Range> uncovered_ranges() const {
    std::vector<Range> rs;
    for (size_t r = 0; r < cursor_.size(); ++r)
      if (end_[r] > cursor_[r]) rs.push_back({cursor_[r], end_[r] - cursor_[r]});
    for (const auto& o : outstanding_) rs.insert(rs.end(), o.begin(), o.end());
    rs.insert(rs.end(), reclaimed_.begin(), reclaimed_.end());
    std::sort(rs.begin(), rs.end());
    std::vector<Range> merged;
    for (const auto& x : rs) {
      if (!merged.empty() && merged.back().first + merged.back().second >= x.first) {
        const int64_t e = std::max(merged.back().first + merged.back().second, x.first + x.second);
        merged.back().second = e - merged.back().first;
      } else {
        merged.push_back(x);
      }
    }
    return merged;
  }

  static ChunkPool from_coverage(int64_t epoch, int64_t total, int world,
                                 const std::vector<Range>& uncovered) {
    std::vector<int64_t> spans(world, 0);
    spans.back() = total;
    ChunkPool p(epoch, total, spans);
    p.cursor_ = p.end_;  // every span consumed; only the holes remain
    std::vector<Range> u = uncovered;
    std::sort(u.begin(), u.end());
    int64_t holes = 0;
    for (const auto& x : u) {
      p.reclaimed_.push_back(x);
      holes += x.second;
    }
    p.completed_ = total - holes;
    return p;
  }

  double epoch_elapsed_ms() const {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0_).count();
  }
  int64_t completed() const { return completed_; }
  int64_t epoch() const { return epoch_; }
  int64_t total() const { return total_; }
  int world() const { return (int)cursor_.size(); }
  std::vector<int64_t> done_samples() const { return done_; }

 private:
  void check_rank(int rank) const {
    if (rank < 0 || rank >= (int)cursor_.size()) throw std::out_of_range("chunk pool: rank out of range");
  }
  int64_t epoch_, total_;
  std::vector<int64_t> start_, cursor_, end_;
  std::deque<Range> reclaimed_;
  std::vector<std::deque<Range>> outstanding_;
  std::vector<int64_t> done_;
  int64_t completed_ = 0;
  std::chrono::steady_clock::time_point t0_;
};

}  // namespace

void register_chunk_pool(py::module& m) {
  py::class_<ChunkPool>(m, "ChunkPool")
      .def(py::init<int64_t, int64_t, const std::vector<int64_t>&>(), py::arg("epoch"),
           py::arg("total"), py::arg("spans"))
      .def("residue", &ChunkPool::residue)
      .def("reservation", &ChunkPool::reservation)
      .def("remaining", &ChunkPool::remaining)
      .def("in_flight", &ChunkPool::in_flight)
      .def("is_epoch_done", &ChunkPool::is_epoch_done)
      .def("take_chunk", &ChunkPool::take_chunk, py::arg("size"), py::arg("rank"))
      .def("rollback_take", &ChunkPool::rollback_take)
      .def("mark_completed", &ChunkPool::mark_completed)
      .def("forfeit", &ChunkPool::forfeit)
      .def("uncovered_ranges", &ChunkPool::uncovered_ranges)
      .def_static("from_coverage", &ChunkPool::from_coverage)
      .def("epoch_elapsed_ms", &ChunkPool::epoch_elapsed_ms)
      .def_property_readonly("completed", &ChunkPool::completed)
      .def_property_readonly("epoch", &ChunkPool::epoch)
      .def_property_readonly("total", &ChunkPool::total)
      .def_property_readonly("world", &ChunkPool::world)
      .def("done_samples", &ChunkPool::done_samples);
}

}  // namespace rt
}  // namespace flodl
