// ElChe: the heterogeneous-DDP cadence balancer (native).
//
// Behaviour follows floDl's ElChe (flodl/src/distributed/el_che.rs,
// docs/ddp/03-internals.md:54-65):
//  * every rank runs `batch_counts[r]` batches per averaging window; the
//    anchor rank (the slowest) runs `anchor` batches, faster ranks
//    proportionally more: round(anchor * slow_ms / ms_r), speed ratio capped
//    at 64. With explicit partition ratios the counts follow the ratios and
//    measured speeds never rebalance them.
//  * per-rank ms/batch is the mean of a ring of the last 5 readings; a rank
//    that reports nothing 5 times in a row has its ring cleared;
//  * anchor election (slow cohort within 15% of the slowest; the current
//    anchor survives unless a challenger is 10% slower; lowest index breaks
//    ties) runs for the first pick and from the Stable phase on. A pinned
//    anchor (speed prior, device prior, partition ratios) that never reports
//    is dropped after 5 empty reports (dead-window escape);
//  * window pressure: overhead = (reduce + fill) / (anchor * marginal +
//    reduce + fill) on the anchor rank; above the target (twice the target
//    during Warmup, never on the first report) a grow to ceil(anchor * min(
//    overhead / target, 2)) is PROPOSED, not applied. The convergence
//    guard's verdict commits it (Stable), vetoes it (SuppressGrowth) or
//    discards it (NudgeDown); a veto or discard latches growth off until 5
//    consecutive Stable verdicts re-arm it. Growth is off when the window
//    cap (one epoch of batches) binds and in Sync mode;
//  * counts change only outside a 5% dead zone (callback slack bypasses it),
//    by at most max_batch_diff per update, and are scaled down to the
//    window cap with the rounding remainder given to the fastest rank;
//  * phases: Probe (no report) -> Warmup -> Stable (5 reports) -> Mature (20);
//  * to_state / restore_from_state carry anchor, anchor rank, smoothed
//    ms/batch, phase and calibration count across a checkpoint.
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
constexpr int kRearmStable = 5;
constexpr int kStableAfter = 5;
constexpr int kMatureAfter = 20;
constexpr size_t kShareWindow = 10;

enum class Phase { kProbe = 0, kWarmup = 1, kStable = 2, kMature = 3 };

const char* phase_name(Phase p) {
  switch (p) {
    case Phase::kProbe: return "probe";
    case Phase::kWarmup: return "warmup";
    case Phase::kStable: return "stable";
    case Phase::kMature: return "mature";
  }
  return "probe";
}

Phase phase_from(const std::string& s) {
  if (s == "warmup") return Phase::kWarmup;
  if (s == "stable") return Phase::kStable;
  if (s == "mature") return Phase::kMature;
  return Phase::kProbe;
}

class ElChe {
 public:
  ElChe(int world, int anchor)
      : world_(world), anchor_(std::max(1, anchor)), min_anchor_(std::max(1, anchor)),
        counts_(world, std::max(1, anchor)), ms_(world), zero_reports_(world, 0),
        slack_(world, 0.0), fill_(world, 0.0) {
    if (world < 1) throw std::runtime_error("ElChe: world_size must be >= 1");
  }

  // ------------------------------------------------------------ configuration
  void set_overhead_target(double t) { overhead_target_ = std::min(0.5, std::max(0.01, t)); }
  void set_max_anchor(int m) {
    max_anchor_ = std::max(1, m);
    if (min_anchor_ > max_anchor_) min_anchor_ = max_anchor_;
    anchor_ = std::min(std::max(anchor_, min_anchor_), max_anchor_);
  }
  void set_min_anchor(int m) {
    min_anchor_ = std::min(std::max(1, m), max_anchor_);
    anchor_ = std::max(anchor_, min_anchor_);
  }
  void set_max_batch_diff(int d) { max_batch_diff_ = d; }
  void set_max_total(int t) { max_total_ = std::max(0, t); }
  void set_growth_applicable(bool b) { growth_applicable_ = b; }
  // Prior: rank `slow_rank` is `ratio` times slower than the others.
  void set_speed_ratio(int slow_rank, double ratio) {
    check_rank(slow_rank);
    anchor_rank_ = slow_rank;
    const double r = std::min(std::max(ratio, 1.0), kMaxSpeedRatio);
    for (int q = 0; q < world_; ++q)
      counts_[q] = q == slow_rank ? anchor_ : std::max(1, (int)std::lround(anchor_ * r));
  }
  void set_initial_anchor(int r) {
    check_rank(r);
    anchor_rank_ = r;
  }
  // Device prior: one spec score per rank (higher = faster hardware); the
  // lowest score (lowest index on ties) becomes the pinned cold-start anchor.
  void set_device_prior(const std::vector<double>& scores) {
    if ((int)scores.size() != world_) return;
    int best = 0;
    for (int r = 1; r < world_; ++r)
      if (scores[r] < scores[best]) best = r;
    anchor_rank_ = best;
  }
  // Explicit per-rank shares (sum ~ 1): the smallest share is the anchor and
  // counts follow the ratios; automatic rebalancing is off.
  void set_partition_ratios(const std::vector<double>& ratios) {
    if ((int)ratios.size() != world_)
      throw std::runtime_error("ElChe: partition_ratios needs one entry per rank");
    double sum = 0.0;
    for (double v : ratios) {
      if (!(v > 0.0) || !std::isfinite(v))
        throw std::runtime_error("ElChe: partition_ratios must be positive and finite");
      sum += v;
    }
    if (std::fabs(sum - 1.0) > 0.01)
      throw std::runtime_error("ElChe: partition_ratios must sum to ~1.0");
    ratios_ = ratios;
    int lo = 0;
    for (int r = 1; r < world_; ++r)
      if (ratios[r] < ratios[lo]) lo = r;
    anchor_rank_ = lo;
    counts_from_ratios();
  }
  void apply_callback_slack(const std::vector<double>& s) {
    if ((int)s.size() == world_) slack_ = s;
  }
  void set_window_fill_ms(const std::vector<double>& f) {
    if ((int)f.size() == world_) fill_ = f;
  }

  // ------------------------------------------------------------ queries
  int batches(int r) const { return counts_.at(r); }
  std::vector<int> batch_counts() const { return counts_; }
  int anchor() const { return anchor_; }
  int anchor_rank() const { return anchor_rank_; }
  int total_batches() const { return std::accumulate(counts_.begin(), counts_.end(), 0); }
  int calibrations() const { return calibrations_; }
  bool is_calibrated() const { return calibrated_; }
  bool has_speed_hint() const {
    for (int r = 1; r < world_; ++r)
      if (counts_[r] != counts_[0]) return true;
    return false;
  }
  std::string phase() const { return phase_name(phase_); }
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
  int proposed_anchor() const { return proposed_; }
  bool growth_enabled() const { return growth_enabled_; }
  bool window_cap_binding() const { return cap_binding_; }
  double anchor_wall_ms() const {
    return calibrated_ && anchor_rank_ >= 0 ? anchor_ * smoothed_ms(anchor_rank_) : 0.0;
  }
  // Per-rank share of the recent windows' batch counts (sums to 1).
  std::vector<double> recent_batch_share() const {
    std::vector<double> s(world_, 0.0);
    double tot = 0.0;
    if (share_.empty()) {
      for (int r = 0; r < world_; ++r) s[r] = counts_[r];
    } else {
      for (const auto& c : share_)
        for (int r = 0; r < world_; ++r) s[r] += c[r];
    }
    for (double v : s) tot += v;
    for (auto& v : s) v = tot > 0.0 ? v / tot : 1.0 / world_;
    return s;
  }

  // ------------------------------------------------------------ timing feed
  // wall_ms[r]: compute wall time of rank r in the window; actual[r]: batches
  // it ran; sync_ms: time of the averaging collective.
  void report_timing(const std::vector<double>& wall_ms, const std::vector<int>& actual,
                     double sync_ms) {
    if ((int)wall_ms.size() != world_ || (int)actual.size() != world_)
      throw std::runtime_error("ElChe::report_timing: one entry per rank required");
    for (int r = 0; r < world_; ++r) {
      if (actual[r] > 0 && wall_ms[r] > 0.0 && std::isfinite(wall_ms[r])) {
        auto& q = ms_[r];
        q.push_back(wall_ms[r] / actual[r]);
        while (q.size() > kTrustWindow) q.pop_front();
        zero_reports_[r] = 0;
      } else if (++zero_reports_[r] >= (int)kTrustWindow) {
        ms_[r].clear();
      }
    }
    if (anchor_rank_ < 0 || phase_ >= Phase::kStable) {
      const int e = elect();
      if (e >= 0) anchor_rank_ = e;
    }
    if (anchor_rank_ < 0) return;
    double slow = smoothed_ms(anchor_rank_);
    if (slow <= 0.0) {
      // dead-window escape: a pinned anchor that never reports is dropped
      if (zero_reports_[anchor_rank_] >= (int)kTrustWindow) {
        const int e = elect();
        if (e >= 0) {
          anchor_rank_ = e;
          slow = smoothed_ms(e);
        }
      }
      if (slow <= 0.0) return;
    }
    proposed_ = 0;
    if (phase_ >= Phase::kStable || (phase_ == Phase::kWarmup && calibrations_ >= 1))
      proposed_ = propose(sync_ms);
    std::fill(fill_.begin(), fill_.end(), 0.0);
    recompute(slow);
    share_.push_back(counts_);
    while (share_.size() > kShareWindow) share_.pop_front();
    calibrated_ = true;
    ++calibrations_;
    if (phase_ == Phase::kProbe) phase_ = Phase::kWarmup;
    if (phase_ == Phase::kWarmup && calibrations_ >= kStableAfter) phase_ = Phase::kStable;
    if (phase_ == Phase::kStable && calibrations_ >= kMatureAfter) phase_ = Phase::kMature;
  }

  // ------------------------------------------------------------ verdicts
  void commit_proposed_anchor() {
    if (++consecutive_stable_ >= kRearmStable) growth_enabled_ = true;
    if (proposed_ > 0) {
      anchor_ = proposed_;
      proposed_ = 0;
      refresh();
    }
  }
  void veto_proposed_growth() {
    proposed_ = 0;
    consecutive_stable_ = 0;
    growth_enabled_ = false;
  }
  void discard_proposed_anchor() { veto_proposed_growth(); }
  // "stable" (commit, then optionally relax up by one), "suppress" (veto) or
  // "nudge" (discard, then scale the anchor down by `factor`).
  void apply_verdict(const std::string& kind, double factor, bool relax_up) {
    if (kind == "stable") {
      commit_proposed_anchor();
      if (relax_up) relax_anchor_up();
    } else if (kind == "suppress") {
      veto_proposed_growth();
    } else if (kind == "nudge") {
      discard_proposed_anchor();
      nudge_anchor_down(factor);
    } else {
      throw std::runtime_error("ElChe::apply_verdict: kind must be stable, suppress or nudge");
    }
  }
  // Divergence is a stronger signal than the overhead floor: min_anchor is
  // bypassed (the anchor may reach 1).
  void nudge_anchor_down(double factor) {
    if (!std::isfinite(factor)) return;
    const int n = (int)std::ceil(anchor_ * std::min(1.0, std::max(0.1, factor)));
    anchor_ = std::max(1, std::min(anchor_, n));
    refresh();
  }
  void relax_anchor_up() {
    if (anchor_ >= max_anchor_) return;
    if (max_batch_diff_ > 0) {
      double mx = 0.0, mn = 0.0;
      for (int r = 0; r < world_; ++r) {
        const double m = smoothed_ms(r);
        mx = std::max(mx, m);
        if (m > 0.0 && (mn == 0.0 || m < mn)) mn = m;
      }
      if (mx > 0.0 && mn > 0.0) {
        const int next = anchor_ + 1;
        const int fast = std::max(1, (int)std::lround(next * mx / mn));
        if (fast - next > max_batch_diff_) return;
      }
    }
    anchor_ += 1;
    refresh();
  }

  std::vector<int> clamp_total(int max_total) const {
    std::vector<int> out = counts_;
    const int tot = std::accumulate(out.begin(), out.end(), 0);
    if (tot <= max_total || max_total <= 0) return out;
    const double f = (double)max_total / tot;
    int used = 0;
    for (auto& v : out) {
      v = std::max(1, (int)std::floor(v * f));
      used += v;
    }
    for (auto& v : out) {
      if (used >= max_total) break;
      ++v;
      ++used;
    }
    return out;
  }

  // ------------------------------------------------------------ checkpoint state
  py::dict to_state() const {
    py::dict d;
    d["anchor"] = anchor_;
    d["anchor_rank"] = anchor_rank_ >= 0 ? py::object(py::int_(anchor_rank_)) : py::none();
    d["smoothed_ms_per_batch"] = ms_per_batch();
    d["phase"] = phase();
    d["calibration_count"] = calibrations_;
    return d;
  }
  void restore_from_state(const py::dict& d) {
    auto ms = d["smoothed_ms_per_batch"].cast<std::vector<double>>();
    if ((int)ms.size() != world_)
      throw std::runtime_error("ElChe::restore_from_state: the snapshot's world size (" +
                               std::to_string(ms.size()) + ") differs from this world (" +
                               std::to_string(world_) + ")");
    anchor_ = std::max(1, d["anchor"].cast<int>());
    anchor_rank_ = d["anchor_rank"].is_none() ? -1 : d["anchor_rank"].cast<int>();
    phase_ = phase_from(d["phase"].cast<std::string>());
    calibrations_ = d["calibration_count"].cast<int>();
    calibrated_ = false;
    for (int r = 0; r < world_; ++r) {
      ms_[r].clear();
      if (ms[r] > 0.0) {
        ms_[r].push_back(ms[r]);  // the mean seeds the window; new readings refill it
        calibrated_ = true;
      }
    }
    if (calibrated_ && anchor_rank_ >= 0 && smoothed_ms(anchor_rank_) > 0.0)
      recompute(smoothed_ms(anchor_rank_));
  }

 private:
  void check_rank(int r) const {
    if (r < 0 || r >= world_) throw std::runtime_error("ElChe: rank out of range");
  }

  int elect() const {
    double mx = 0.0;
    for (int r = 0; r < world_; ++r) mx = std::max(mx, smoothed_ms(r));
    if (mx <= 0.0) return -1;
    std::vector<int> cohort;
    for (int r = 0; r < world_; ++r)
      if (smoothed_ms(r) >= mx * (1.0 - kCohortBand)) cohort.push_back(r);
    if (cohort.size() == 1) return cohort[0];
    if (anchor_rank_ >= 0 && std::find(cohort.begin(), cohort.end(), anchor_rank_) != cohort.end()) {
      const double cur = smoothed_ms(anchor_rank_);
      int best = -1;
      double best_ms = 0.0;
      for (int r : cohort)
        if (r != anchor_rank_ && smoothed_ms(r) > best_ms) {
          best = r;
          best_ms = smoothed_ms(r);
        }
      if (best >= 0 && best_ms > cur * (1.0 + kDominanceMargin)) return best;
      return anchor_rank_;
    }
    return *std::min_element(cohort.begin(), cohort.end());
  }

  // Window-pressure grow proposal (0: none).
  int propose(double sync_ms) {
    if (!growth_applicable_ || !growth_enabled_ || cap_binding_ || anchor_rank_ < 0) return 0;
    const double marginal = smoothed_ms(anchor_rank_);
    if (marginal <= 0.0) return 0;
    const double fixed = std::max(0.0, sync_ms) + std::max(0.0, fill_[anchor_rank_]);
    const double denom = anchor_ * marginal + fixed;
    if (fixed <= 0.0 || denom <= 0.0) return 0;
    const double overhead = fixed / denom;
    last_overhead_ = overhead;
    const double fire = phase_ >= Phase::kStable ? overhead_target_ : overhead_target_ * kGrowthStepCap;
    if (overhead <= fire) return 0;
    const double scale = std::min(kGrowthStepCap, overhead / overhead_target_);
    const int next = std::min(max_anchor_, std::max(min_anchor_, (int)std::ceil(anchor_ * scale)));
    return next > anchor_ ? next : 0;
  }

  void refresh() {
    if (!ratios_.empty()) {
      counts_from_ratios();
      return;
    }
    const double slow = anchor_rank_ >= 0 ? smoothed_ms(anchor_rank_) : 0.0;
    if (slow > 0.0) recompute(slow);
  }

  void counts_from_ratios() {
    const double lo = ratios_[anchor_rank_ >= 0 ? anchor_rank_ : 0];
    for (int r = 0; r < world_; ++r)
      counts_[r] = std::max(1, (int)std::lround(anchor_ * ratios_[r] / lo));
    cap(counts_);
  }

  void recompute(double slow) {
    if (!ratios_.empty()) {
      counts_from_ratios();
      std::fill(slack_.begin(), slack_.end(), 0.0);
      return;
    }
    for (int r = 0; r < world_; ++r) {
      const double ms = smoothed_ms(r);
      int target = (ms <= 0.0 || std::fabs(ms - slow) < 1e-6)
                       ? anchor_
                       : std::max(1, (int)std::lround(anchor_ * std::min(slow / ms, kMaxSpeedRatio)));
      const int slack = (slack_[r] > 0.0 && ms > 0.0) ? (int)std::ceil(slack_[r] / ms) : 0;
      target = std::max(1, target - slack);
      const int cur = counts_[r];
      if (std::fabs((double)target - cur) > cur * 0.05 || !calibrated_ || slack > 0) {
        int v = target;
        if (max_batch_diff_ > 0 && calibrated_)
          v = target > cur ? std::min(cur + max_batch_diff_, target)
                           : std::max(std::max(cur - max_batch_diff_, target), 1);
        counts_[r] = v;
      }
    }
    cap(counts_);
    std::fill(slack_.begin(), slack_.end(), 0.0);
  }

  // Scale the window down to max_total (one epoch of batches); the rounding
  // remainder goes to the rank with the largest count.
  void cap(std::vector<int>& c) {
    cap_binding_ = false;
    if (max_total_ <= 0) return;
    const int tot = std::accumulate(c.begin(), c.end(), 0);
    if (tot <= max_total_) return;
    cap_binding_ = true;
    const double f = (double)max_total_ / tot;
    int used = 0;
    for (auto& v : c) {
      v = std::max(1, (int)std::floor(v * f));
      used += v;
    }
    if (used < max_total_) {
      auto it = std::max_element(c.begin(), c.end());
      *it += max_total_ - used;
    }
  }

  int world_;
  int anchor_;
  int anchor_rank_ = -1;
  int max_anchor_ = 1000;
  int min_anchor_;
  std::vector<int> counts_;
  std::vector<std::deque<double>> ms_;
  std::vector<int> zero_reports_;
  std::vector<double> slack_;
  std::vector<double> fill_;
  std::vector<double> ratios_;
  std::deque<std::vector<int>> share_;
  double overhead_target_ = 0.05;
  int max_batch_diff_ = 0;
  int max_total_ = 0;
  bool growth_applicable_ = true;
  bool growth_enabled_ = true;
  int consecutive_stable_ = 0;
  bool cap_binding_ = false;
  bool calibrated_ = false;
  int calibrations_ = 0;
  int proposed_ = 0;
  Phase phase_ = Phase::kProbe;
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
      .def("set_device_prior", &ElChe::set_device_prior)
      .def("set_partition_ratios", &ElChe::set_partition_ratios)
      .def("apply_callback_slack", &ElChe::apply_callback_slack)
      .def("set_window_fill_ms", &ElChe::set_window_fill_ms)
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
      .def("proposed_anchor", &ElChe::proposed_anchor)
      .def("growth_enabled", &ElChe::growth_enabled)
      .def("window_cap_binding", &ElChe::window_cap_binding)
      .def("anchor_wall_ms", &ElChe::anchor_wall_ms)
      .def("recent_batch_share", &ElChe::recent_batch_share)
      .def("report_timing", &ElChe::report_timing, py::arg("wall_ms"), py::arg("actual_batches"),
           py::arg("sync_ms"))
      .def("commit_proposed_anchor", &ElChe::commit_proposed_anchor)
      .def("veto_proposed_growth", &ElChe::veto_proposed_growth)
      .def("discard_proposed_anchor", &ElChe::discard_proposed_anchor)
      .def("apply_verdict", &ElChe::apply_verdict, py::arg("kind"), py::arg("factor") = 1.0,
           py::arg("relax_up") = false)
      .def("nudge_anchor_down", &ElChe::nudge_anchor_down)
      .def("relax_anchor_up", &ElChe::relax_anchor_up)
      .def("clamp_total", &ElChe::clamp_total)
      .def("to_state", &ElChe::to_state)
      .def("restore_from_state", &ElChe::restore_from_state);
}

}  // namespace rt
}  // namespace flodl
