// ElChe: the heterogeneous-DDP cadence balancer (native).
//
// Behaviour follows floDl's ElChe (flodl/src/distributed/el_che.rs:160-1560,
// docs/ddp/03-internals.md:54-65):
//  * every rank runs `batch_counts[r]` batches per averaging window; the
//    slowest rank (the anchor) runs `anchor` batches, faster ranks
//    proportionally more: round(anchor * slow_ms / ms_r), speed ratio capped;
//  * per-rank ms/batch is the mean of a ring buffer of the last 5 readings;
//  * anchor election: among ranks within 15% of the slowest (the cohort), the
//    current anchor is only replaced by a challenger at least 10% slower, and
//    only once calibration reached the Stable phase;
//  * counts change only outside a 5% dead zone, by at most max_batch_diff per
//    update, and their sum is scaled down to max_total (one epoch) if set;
//  * overhead auto-tune: overhead = sync / (wall - sync); above the target the
//    anchor grows by ceil(anchor * overhead / target) (at most x2 per step,
//    during Warmup only when the signal exceeds 2x the target); below
//    target/2 it shrinks by one; clamped to [min_anchor, max_anchor];
//  * phases: Probe (no timing yet) -> Warmup (< 5 calibrations) -> Stable ->
//    Mature (>= 20 calibrations).
#include "runtime.h"

#include <algorithm>
#include <cmath>
#include <deque>
#include <numeric>
#include <stdexcept>

namespace flodl {
namespace rt {

namespace {

constexpr double kCohortBand = 0.15;
constexpr double kDominanceMargin = 0.10;
constexpr size_t kTrustWindow = 5;
constexpr double kMaxSpeedRatio = 64.0;
constexpr double kGrowthStepCap = 2.0;
constexpr int kStableAfter = 5;
constexpr int kMatureAfter = 20;

class ElChe {
 public:
  ElChe(int world, int anchor)
      : world_(world), anchor_(std::max(1, anchor)), counts_(world, std::max(1, anchor)),
        ms_(world), slack_(world, 0.0) {
    if (world < 1) throw std::runtime_error("ElChe: world_size must be >= 1");
  }

  // configuration
  void set_overhead_target(double t) { overhead_target_ = t; }
  void set_max_anchor(int m) { max_anchor_ = m; }
  void set_min_anchor(int m) { min_anchor_ = std::max(1, m); }
  void set_max_batch_diff(int d) { max_batch_diff_ = d; }
  void set_max_total(int t) { max_total_ = t; }
  void set_growth_applicable(bool b) { growth_applicable_ = b; }
  void set_speed_ratio(int slow_rank, double ratio) {
    // A prior: rank `slow_rank` is `ratio` times slower than the others.
    anchor_rank_ = slow_rank;
    for (int r = 0; r < world_; ++r)
      counts_[r] = r == slow_rank ? anchor_
                                  : std::max(1, (int)std::lround(anchor_ * std::min(ratio, kMaxSpeedRatio)));
    speed_hint_ = true;
  }
  void set_initial_anchor(int r) { anchor_rank_ = r; }
  void apply_callback_slack(const std::vector<double>& s) {
    if ((int)s.size() == world_) slack_ = s;
  }

  // queries
  int batches(int r) const { return counts_.at(r); }
  std::vector<int> batch_counts() const { return counts_; }
  int anchor() const { return anchor_; }
  int anchor_rank() const { return anchor_rank_; }
  int total_batches() const { return std::accumulate(counts_.begin(), counts_.end(), 0); }
  int calibrations() const { return calibrations_; }
  bool is_calibrated() const { return calibrations_ > 0; }
  bool has_speed_hint() const { return speed_hint_; }
  std::string phase() const {
    if (calibrations_ == 0) return "probe";
    if (calibrations_ < kStableAfter) return "warmup";
    if (calibrations_ < kMatureAfter) return "stable";
    return "mature";
  }
  double smoothed_ms(int r) const {
    const auto& q = ms_.at(r);
    if (q.empty()) return 0.0;
    return std::accumulate(q.begin(), q.end(), 0.0) / (double)q.size();
  }
  std::vector<double> ms_per_batch() const {
    std::vector<double> out(world_);
    for (int r = 0; r < world_; ++r) out[r] = smoothed_ms(r);
    return out;
  }
  double last_overhead() const { return last_overhead_; }

  // wall_ms[r]: compute wall time of rank r in the window; actual[r]: batches
  // it ran; sync_ms: time of the averaging collective.
  void report_timing(const std::vector<double>& wall_ms, const std::vector<int>& actual,
                     double sync_ms) {
    if ((int)wall_ms.size() != world_ || (int)actual.size() != world_)
      throw std::runtime_error("ElChe::report_timing: one entry per rank required");
    for (int r = 0; r < world_; ++r) {
      if (actual[r] <= 0 || wall_ms[r] <= 0.0) continue;
      auto& q = ms_[r];
      q.push_back(wall_ms[r] / actual[r]);
      while (q.size() > kTrustWindow) q.pop_front();
    }
    ++calibrations_;
    elect_anchor();
    const double slow = smoothed_ms(anchor_rank_);
    // overhead auto-tune on the anchor's wall time
    const double aw = wall_ms[anchor_rank_];
    if (growth_applicable_ && aw > sync_ms && sync_ms >= 0.0) {
      const double overhead = sync_ms / std::max(1e-9, aw - sync_ms);
      last_overhead_ = overhead;
      const bool warm = calibrations_ < kStableAfter;
      if (overhead > overhead_target_ && (!warm || overhead > kGrowthStepCap * overhead_target_)) {
        const double scale = std::min(kGrowthStepCap, overhead / overhead_target_);
        int proposed = (int)std::ceil(anchor_ * scale);
        if (proposed > anchor_) anchor_ = proposed;
      } else if (overhead < overhead_target_ / 2.0 && anchor_ > min_anchor_) {
        anchor_ -= 1;
      }
      if (max_anchor_ > 0) anchor_ = std::min(anchor_, max_anchor_);
      anchor_ = std::max(anchor_, min_anchor_);
    }
    recompute(slow);
    calibrated_ = true;
  }

  void nudge_anchor_down(double factor) {
    anchor_ = std::max(min_anchor_, (int)std::floor(anchor_ * factor));
    recompute(smoothed_ms(anchor_rank_));
  }
  void relax_anchor_up() {
    anchor_ += 1;
    if (max_anchor_ > 0) anchor_ = std::min(anchor_, max_anchor_);
    recompute(smoothed_ms(anchor_rank_));
  }

  std::vector<int> clamp_total(int max_total) const {
    std::vector<int> out = counts_;
    scale_to(out, max_total);
    return out;
  }

 private:
  void elect_anchor() {
    double slowest = -1.0;
    int slowest_rank = anchor_rank_;
    for (int r = 0; r < world_; ++r) {
      double m = smoothed_ms(r);
      if (m > slowest) {
        slowest = m;
        slowest_rank = r;
      }
    }
    if (slowest <= 0.0) return;
    if (calibrations_ == 1 && !speed_hint_) {
      anchor_rank_ = slowest_rank;  // initial pick
      return;
    }
    if (calibrations_ <= kStableAfter) return;  // lock the initial pick through warmup
    const double cur = smoothed_ms(anchor_rank_);
    const bool cur_in_cohort = cur >= (1.0 - kCohortBand) * slowest;
    if (!cur_in_cohort || slowest >= cur * (1.0 + kDominanceMargin)) anchor_rank_ = slowest_rank;
  }

  void recompute(double slow_ms) {
    for (int r = 0; r < world_; ++r) {
      const double ms = smoothed_ms(r);
      int target;
      if (ms <= 0.0 || std::fabs(ms - slow_ms) < 1e-6)
        target = anchor_;
      else
        target = std::max(1, (int)std::lround(anchor_ * std::min(slow_ms / ms, kMaxSpeedRatio)));
      int slack_batches = 0;
      if (slack_[r] > 0.0 && ms > 0.0) slack_batches = (int)std::ceil(slack_[r] / ms);
      target = std::max(1, target - slack_batches);
      const int cur = counts_[r];
      const double diff = std::fabs((double)target - cur);
      if (diff > cur * 0.05 || !calibrated_ || slack_batches > 0) {
        int v = target;
        if (max_batch_diff_ > 0 && calibrated_) {
          v = target > cur ? std::min(cur + max_batch_diff_, target)
                           : std::max(std::max(cur - max_batch_diff_, target), 1);
        }
        counts_[r] = v;
      }
    }
    std::fill(slack_.begin(), slack_.end(), 0.0);
    if (max_total_ > 0) scale_to(counts_, max_total_);
  }

  static void scale_to(std::vector<int>& c, int max_total) {
    const int tot = std::accumulate(c.begin(), c.end(), 0);
    if (tot <= max_total || tot == 0) return;
    const double f = (double)max_total / tot;
    for (auto& v : c) v = std::max(1, (int)std::floor(v * f));
  }

  int world_;
  int anchor_;
  int anchor_rank_ = 0;
  std::vector<int> counts_;
  std::vector<std::deque<double>> ms_;
  std::vector<double> slack_;
  double overhead_target_ = 0.10;
  int max_anchor_ = 0;
  int min_anchor_ = 1;
  int max_batch_diff_ = 0;
  int max_total_ = 0;
  bool growth_applicable_ = true;
  bool speed_hint_ = false;
  bool calibrated_ = false;
  int calibrations_ = 0;
  double last_overhead_ = 0.0;
};

}  // namespace

void register_elche(py::module& m) {
  py::class_<ElChe>(m, "ElChe")
      .def(py::init<int, int>(), py::arg("world_size"), py::arg("anchor"))
      .def("set_overhead_target", &ElChe::set_overhead_target)
      .def("set_max_anchor", &ElChe::set_max_anchor)
      .def("set_min_anchor", &ElChe::set_min_anchor)
      .def("set_max_batch_diff", &ElChe::set_max_batch_diff)
      .def("set_max_total", &ElChe::set_max_total)
      .def("set_growth_applicable", &ElChe::set_growth_applicable)
      .def("set_speed_ratio", &ElChe::set_speed_ratio)
      .def("set_initial_anchor", &ElChe::set_initial_anchor)
      .def("apply_callback_slack", &ElChe::apply_callback_slack)
      .def("batches", &ElChe::batches)
      .def("batch_counts", &ElChe::batch_counts)
      .def("anchor", &ElChe::anchor)
      .def("anchor_rank", &ElChe::anchor_rank)
      .def("total_batches", &ElChe::total_batches)
      .def("calibrations", &ElChe::calibrations)
      .def("is_calibrated", &ElChe::is_calibrated)
      .def("has_speed_hint", &ElChe::has_speed_hint)
      .def("phase", &ElChe::phase)
      .def("smoothed_ms", &ElChe::smoothed_ms)
      .def("ms_per_batch", &ElChe::ms_per_batch)
      .def("last_overhead", &ElChe::last_overhead)
      .def("report_timing", &ElChe::report_timing, py::arg("wall_ms"), py::arg("actual_batches"),
           py::arg("sync_ms"))
      .def("nudge_anchor_down", &ElChe::nudge_anchor_down)
      .def("relax_anchor_up", &ElChe::relax_anchor_up)
      .def("clamp_total", &ElChe::clamp_total);
}

}  // namespace rt
}  // namespace flodl
