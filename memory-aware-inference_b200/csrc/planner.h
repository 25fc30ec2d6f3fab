// Planner trace core shared by the C ABI (planner.cu) and the model's
// measured ring trace (model.cu).
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <utility>
#include <vector>

namespace si {

// One planner action (PlannerAction, src/planner.rs:39-50).
struct TraceAction {
  uint32_t kind = 0, tier = 0;  // SI_ACT_*, SI_TIER_*
  std::string op, queue, reason, tensors_joined;
  std::vector<std::string> tensors;
  uint64_t bytes = 0, started_ns = 0, ended_ns = 0;
};

// PlannerTrace (src/planner.rs:62-170): actions validated as they are
// recorded against the residency they imply.
struct TraceCore {
  uint32_t mode = 0;
  std::vector<TraceAction> actions;
  uint64_t planned_peak_hbm = 0, observed_peak_hbm = 0, observed_peak_rss = 0;
  bool observed = false;
  std::map<std::pair<uint32_t, std::string>, uint64_t> resident;
  int record(TraceAction a, std::string* err);
};

}  // namespace si

struct si_trace {
  si::TraceCore core;
};
