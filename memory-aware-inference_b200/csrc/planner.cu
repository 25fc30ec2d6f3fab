// Planner traces (host code): PlannerTrace::record and plan_sequential_layers
// (src/planner.rs:62-251) behind the C ABI. The model records measured traces
// of its staging ring with the same core (model.cu, si_model_trace_*).
#include <cstring>
#include <string>

#include "../../include/si_cuda.h"
#include "planner.h"

namespace si {

int fail(si_ctx* ctx, int code, const std::string& msg);

int TraceCore::record(TraceAction a, std::string* err) {
  if (a.tensors.empty()) {
    *err = "planner action must name a tensor";
    return SI_E_INVALID;
  }
  if (a.ended_ns < a.started_ns) {
    *err = "action " + a.op + " ends before it starts";
    return SI_E_INVALID;
  }
  switch (a.kind) {
    case SI_ACT_PREFETCH:
    case SI_ACT_RETAIN: {
      const uint64_t per = a.bytes / a.tensors.size();
      for (const auto& t : a.tensors) resident[{a.tier, t}] = per;
      break;
    }
    case SI_ACT_EXECUTE:
      for (const auto& t : a.tensors)
        if (!resident.count({a.tier, t})) {
          *err = "operation " + a.op + " executes non-resident tensor " + t;
          return SI_E_STATE;
        }
      break;
    case SI_ACT_EVICT:
    case SI_ACT_RELEASE:
      for (const auto& t : a.tensors)
        if (!resident.erase({a.tier, t})) {
          *err = "operation " + a.op + " evicts non-resident tensor " + t;
          return SI_E_STATE;
        }
      break;
    case SI_ACT_WAIT:
      break;
    default:
      *err = "unknown planner action kind " + std::to_string(a.kind);
      return SI_E_INVALID;
  }
  if (a.tier == SI_TIER_HBM && (a.kind == SI_ACT_PREFETCH || a.kind == SI_ACT_RETAIN)) {
    uint64_t cur = 0;
    for (const auto& r : resident)
      if (r.first.first == SI_TIER_HBM) cur += r.second;
    planned_peak_hbm = std::max(planned_peak_hbm, cur);
  }
  a.tensors_joined.clear();
  for (size_t i = 0; i < a.tensors.size(); ++i) a.tensors_joined += (i ? "," : "") + a.tensors[i];
  actions.push_back(std::move(a));
  return SI_OK;
}

}  // namespace si

extern "C" {

si_trace* si_trace_create(uint32_t mode) {
  auto* t = new si_trace();
  t->core.mode = mode;
  return t;
}

void si_trace_destroy(si_trace* t) { delete t; }

int si_trace_record(si_trace* t, const si_trace_action* a) {
  if (!t || !a || !a->operation_id) return si::fail(nullptr, SI_E_INVALID, "invalid trace arguments");
  si::TraceAction x;
  x.kind = a->kind;
  x.tier = a->tier;
  x.op = a->operation_id;
  x.queue = a->queue ? a->queue : "";
  x.reason = a->reason ? a->reason : "";
  x.bytes = a->bytes;
  x.started_ns = a->started_ns;
  x.ended_ns = a->ended_ns;
  if (a->tensor_ids && *a->tensor_ids) {
    std::string s = a->tensor_ids, cur;
    for (char ch : s) {
      if (ch == ',') {
        x.tensors.push_back(cur);
        cur.clear();
      } else {
        cur += ch;
      }
    }
    x.tensors.push_back(cur);
  }
  std::string err;
  const int rc = t->core.record(std::move(x), &err);
  return rc ? si::fail(nullptr, rc, err) : SI_OK;
}

int si_trace_count(const si_trace* t, uint64_t* n) {
  if (!t || !n) return SI_E_INVALID;
  *n = t->core.actions.size();
  return SI_OK;
}

int si_trace_action_at(const si_trace* t, uint64_t i, si_trace_action* out) {
  if (!t || !out || i >= t->core.actions.size()) return si::fail(nullptr, SI_E_INVALID, "trace index out of range");
  const si::TraceAction& a = t->core.actions[i];
  out->kind = a.kind;
  out->tier = a.tier;
  out->operation_id = a.op.c_str();
  out->tensor_ids = a.tensors_joined.c_str();
  out->bytes = a.bytes;
  out->started_ns = a.started_ns;
  out->ended_ns = a.ended_ns;
  out->queue = a.queue.c_str();
  out->reason = a.reason.c_str();
  return SI_OK;
}

int si_trace_summary(const si_trace* t, si_trace_summary_info* out) {
  if (!t || !out) return SI_E_INVALID;
  std::memset(out, 0, sizeof(*out));
  out->mode = t->core.mode;
  out->actions = t->core.actions.size();
  out->planned_peak_hbm_bytes = t->core.planned_peak_hbm;
  out->observed = t->core.observed ? 1 : 0;
  out->observed_peak_hbm_bytes = t->core.observed_peak_hbm;
  out->observed_peak_rss_bytes = t->core.observed_peak_rss;
  for (const auto& r : t->core.resident) {
    if (r.first.first == SI_TIER_HBM) {
      out->resident_hbm_tensors++;
      out->resident_hbm_bytes += r.second;
    }
  }
  return SI_OK;
}

int si_plan_sequential_layers(uint32_t layers, const char* const* operation_ids, const uint32_t* tensor_counts,
                              const char* const* tensor_ids, const uint64_t* tensor_bytes, uint64_t budget_bytes,
                              si_trace** out) {
  if (!out) return SI_E_INVALID;
  *out = nullptr;
  if (layers == 0) return si::fail(nullptr, SI_E_INVALID, "layer plan must contain at least one layer");
  if (budget_bytes == 0) return si::fail(nullptr, SI_E_INVALID, "HBM budget must be non-zero");
  if (!operation_ids || !tensor_counts || !tensor_ids || !tensor_bytes)
    return si::fail(nullptr, SI_E_INVALID, "invalid layer plan arguments");
  auto* t = si_trace_create(SI_MODE_LAYER_STREAM);
  uint64_t ts = 0, k = 0;
  std::string err;
  auto bad = [&](int code, const std::string& msg) {
    si_trace_destroy(t);
    return si::fail(nullptr, code, msg);
  };
  for (uint32_t l = 0; l < layers; ++l) {
    const std::string op = operation_ids[l] ? operation_ids[l] : "";
    if (tensor_counts[l] == 0) return bad(SI_E_INVALID, "layer " + op + " has no tensors");
    uint64_t layer_bytes = 0;
    for (uint32_t i = 0; i < tensor_counts[l]; ++i) {
      if (tensor_bytes[k + i] > UINT64_MAX - layer_bytes) return bad(SI_E_INVALID, "layer byte size overflow");
      layer_bytes += tensor_bytes[k + i];
    }
    if (layer_bytes > budget_bytes)
      return bad(SI_E_BUDGET, "layer " + op + " requires " + std::to_string(layer_bytes) + " bytes but budget is " +
                                  std::to_string(budget_bytes));
    si::TraceAction ex;
    ex.kind = SI_ACT_EXECUTE;
    ex.tier = SI_TIER_HBM;
    ex.op = op;
    ex.bytes = layer_bytes;
    ex.started_ns = ex.ended_ns = ts;
    ex.queue = "compute";
    ex.reason = "execute layer with all required tensors resident";
    for (uint32_t i = 0; i < tensor_counts[l]; ++i) {
      si::TraceAction a;
      a.kind = SI_ACT_PREFETCH;
      a.tier = SI_TIER_HBM;
      a.op = op;
      a.tensors = {tensor_ids[k + i] ? tensor_ids[k + i] : ""};
      a.bytes = tensor_bytes[k + i];
      a.started_ns = a.ended_ns = ts;
      a.queue = "transfer";
      a.reason = "make current layer available before execution";
      ex.tensors.push_back(a.tensors[0]);
      if (int rc = t->core.record(std::move(a), &err)) return bad(rc, err);
    }
    if (int rc = t->core.record(ex, &err)) return bad(rc, err);
    ++ts;
    for (uint32_t i = 0; i < tensor_counts[l]; ++i) {
      si::TraceAction a;
      a.kind = SI_ACT_EVICT;
      a.tier = SI_TIER_HBM;
      a.op = op;
      a.tensors = {tensor_ids[k + i] ? tensor_ids[k + i] : ""};
      a.bytes = tensor_bytes[k + i];
      a.started_ns = a.ended_ns = ts;
      a.queue = "transfer";
      a.reason = "release layer before advancing the bounded window";
      if (int rc = t->core.record(std::move(a), &err)) return bad(rc, err);
    }
    ++ts;
    k += tensor_counts[l];
  }
  *out = t;
  return SI_OK;
}

}  // extern "C"
