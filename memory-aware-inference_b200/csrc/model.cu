// Synthetic Qwen3.6-shaped decoder on the CUDA backend: seeded weights in
// pinned host memory, a residency plan inside the HBM budget, a depth-N
// staging ring for the streamed layers, the per-token layer loop, greedy
// generation, and row sharding over a NCCL communicator.
//
// Reference counterparts: Qwen35Runtime (src/qwen35_runtime.rs:1519-2267):
// decode_hidden 1776-1941, logits 2132-2192, decode_token 2229-2246, staging
// 2283-2332; residency selection 1552-1733; planner budget check
// (src/planner.rs:174-251); run_gguf_generation (src/runtime.rs:3560-3614).
#include <unistd.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "comm.h"
#include "common.cuh"
#include "ctx.h"
#include "fault.h"
#include "gguf.h"
#include "planner.h"
#include "kernels.cuh"

#include <nvtx3/nvToolsExt.h>
#include "qmatvec.cuh"
#include "synth.h"

using namespace si;


namespace {

struct RowRange {
  uint64_t begin, end;
};

struct LocalTensor {
  bool present = false;
  uint32_t type = 0;
  uint64_t full_rows = 0, cols = 0, rows = 0;  // rows = local rows
  std::vector<RowRange> ranges;                 // full-tensor rows held locally
  uint64_t offset = 0, bytes = 0;               // inside the packed layer buffer
  float mean = 0.f, stdev = 0.f;                // F32 tensors
};

struct LayerLayout {
  bool gdn = false;
  LocalTensor t[SI_T_COUNT];
  uint64_t bytes = 0;
};

uint64_t row_bytes_of(uint32_t type, uint64_t cols) {
  return type == SI_GGML_TYPE_F32 ? cols * 4 : cols / 256 * block_bytes_of(type);
}

uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

}  // namespace

struct si_model {
  si_ctx* ctx = nullptr;
  si_model_config c{};
  uint64_t seed = 0;
  int n = 1, r = 0;
  // sharded dims
  uint32_t kh_l = 0, vh_l = 0, qh_l = 0, kv_lo = 0, kvh_l = 0, H_l = 0, I_l = 0, V_l = 0;
  std::vector<LayerLayout> layout;  // [layers + 1], globals at index `layers`
  // per-tensor ggml types read from a GGUF file ([layers + 1]); empty: the
  // config's per-role types
  std::vector<std::array<uint32_t, SI_T_COUNT>> ttype;
  std::vector<uint8_t*> host;       // pinned packed layer buffers
  uint8_t* embd_host = nullptr;     // mapped pinned token_embd shard
  uint8_t* embd_dev = nullptr;
  // residency
  std::vector<uint8_t*> dev_layer;  // resident pointer or nullptr (streamed)
  uint8_t* dev_resident = nullptr;
  std::vector<uint32_t> streamed;
  uint32_t depth = 3;
  uint8_t* slot[4] = {nullptr, nullptr, nullptr, nullptr};
  cudaEvent_t copy_done[4] = {}, compute_done[4] = {};
  uint64_t occ_issued = 0, occ_next = 0;  // streamed-layer occurrences
  si_plan_info plan{};
  // state
  std::vector<float*> conv[2];
  std::vector<float*> rec;
  std::vector<uint16_t*> kc, vc;
  std::vector<uint32_t> cached;
  std::vector<uint32_t> conv_parity;
  uint8_t* state_block = nullptr;
  // scratch
  uint8_t* scratch_block = nullptr;
  float *hidden, *slice, *qkv, *z, *ab, *core, *core_full, *z_full, *qg, *kk, *vv, *att,
      *att_full, *gate_full, *gate_l, *act, *act_full, *logits, *logits_full, *rope, *part, *embed, *up;
  uint32_t* d_token;
  unsigned long long *d_key, *d_keys;
  // batched verifier (decode_tokens_many): candidate-major buffers for up to
  // kQmmMaxBatch tokens, inside the scratch block (unsharded models only)
  float *b_hid = nullptr, *b_xn, *b_xg, *b_qkv, *b_z, *b_ab, *b_core, *b_qg, *b_kk, *b_vv, *b_att, *b_act,
        *b_up, *b_logits;
  unsigned long long* b_keys;
  uint32_t *b_ids, *b_tokens;
  uint8_t* b_qmm = nullptr;  // tensor-core batched matvec scratch (digits, tables, panel sums)
  uint64_t b_qmm_bytes = 0;
  uint32_t b_valid = 0;  // candidates whose final hidden states are in b_hid
  // NVLink peer all-gather: every rank's scratch block mapped here (CUDA IPC)
  bool p2p = false;
  void* peer_block[kP2PMaxRanks] = {};
  uint32_t p2p_epoch = 0;
  uint64_t flag_off = 0;
  // in-kernel all-gather of the Q4_K matvecs' outputs (PeerOut): offsets in
  // the scratch block of the CTA ticket, the launch epoch and the exchange
  // words of the hidden and activation vectors (two parity halves each)
  uint64_t xchg_ticket_off = 0, xchg_epoch_off = 0, ll_hidden_off = 0, ll_act_off = 0, ll_core_off = 0, ll_z_off = 0,
           ll_att_off = 0, ll_gate_off = 0;
  // tensor-level retention: of a streamed layer l the packed bytes
  // [0, part_bytes[l]) stay resident at dev_part[l] (the ring copies the rest)
  std::vector<uint64_t> part_bytes;
  std::vector<uint8_t*> dev_part;
  std::vector<float> rope_host;
  bool accounted = false;  // device bytes recorded in the context telemetry
  // measured planner trace (si_model_trace_begin / _end)
  struct TraceRec {
    uint32_t kind;
    int layer;          // layer index; layers = the output head
    int slot;           // ring slot, -1 for a resident layer
    cudaEvent_t e0, e1; // null: at the start of the trace (retained before it)
    uint64_t bytes;
  };
  bool tracing = false;
  std::vector<cudaEvent_t> tr_pool;
  size_t tr_used = 0;
  std::vector<TraceRec> tr_recs;
  cudaEvent_t tr_base = nullptr;
  int slot_layer[4] = {-1, -1, -1, -1};  // layer staged in each ring slot
};

namespace {

// Full tensor shapes of one layer / the globals (qwen35_runtime.rs:419-446,
// 640-657, model.rs:418-441).
void full_spec(const si_model_config& c, bool gdn, bool globals, LayerLayout* L) {
  auto set = [&](int id, uint32_t type, uint64_t rows, uint64_t cols, float mean = 0.f, float sd = 0.f) {
    LocalTensor& t = L->t[id];
    t.present = true;
    t.type = type;
    t.full_rows = rows;
    t.cols = cols;
    t.mean = mean;
    t.stdev = sd;
  };
  const uint64_t H = c.hidden, I = c.intermediate, d = c.gdn_head_dim;
  if (globals) {
    set(SI_T_OUTPUT_NORM, SI_GGML_TYPE_F32, 1, H, 0.f, 0.1f);
    set(SI_T_OUTPUT, c.head_type, c.vocab, H);
    return;  // token_embd is held separately (mapped host memory)
  }
  set(SI_T_ATTN_NORM, SI_GGML_TYPE_F32, 1, H, 0.f, 0.1f);
  set(SI_T_POST_NORM, SI_GGML_TYPE_F32, 1, H, 0.f, 0.1f);
  set(SI_T_FFN_GATE, c.mlp_type, I, H);
  set(SI_T_FFN_UP, c.mlp_type, I, H);
  set(SI_T_FFN_DOWN, c.down_type, H, I);
  if (gdn) {
    const uint64_t proj = (2ull * c.gdn_key_heads + c.gdn_value_heads) * d, vw = uint64_t(c.gdn_value_heads) * d;
    set(SI_T_SSM_QKV, SI_GGML_TYPE_Q4_K, proj, H);
    set(SI_T_SSM_Z, SI_GGML_TYPE_Q4_K, vw, H);
    set(SI_T_SSM_ALPHA, SI_GGML_TYPE_F32, c.gdn_value_heads, H, 0.f, 0.02f);
    set(SI_T_SSM_BETA, SI_GGML_TYPE_F32, c.gdn_value_heads, H, 0.f, 0.02f);
    set(SI_T_SSM_CONV, SI_GGML_TYPE_F32, proj, c.conv_kernel, 0.f, 0.5f);
    set(SI_T_SSM_A, SI_GGML_TYPE_F32, c.gdn_value_heads, 1, 0.f, 0.5f);
    set(SI_T_SSM_DT, SI_GGML_TYPE_F32, c.gdn_value_heads, 1, 0.f, 0.5f);
    set(SI_T_SSM_NORM, SI_GGML_TYPE_F32, 1, d, 1.f, 0.1f);
    set(SI_T_SSM_OUT, SI_GGML_TYPE_Q4_K, H, vw);
  } else {
    const uint64_t qw = uint64_t(c.attn_q_heads) * c.attn_head_dim, kvw = uint64_t(c.attn_kv_heads) * c.attn_head_dim;
    set(SI_T_ATTN_Q, SI_GGML_TYPE_Q4_K, 2 * qw, H);
    set(SI_T_ATTN_K, SI_GGML_TYPE_Q4_K, kvw, H);
    set(SI_T_ATTN_V, SI_GGML_TYPE_Q4_K, kvw, H);
    set(SI_T_ATTN_O, SI_GGML_TYPE_Q4_K, H, qw);
    set(SI_T_ATTN_QNORM, SI_GGML_TYPE_F32, 1, c.attn_head_dim, 0.f, 0.1f);
    set(SI_T_ATTN_KNORM, SI_GGML_TYPE_F32, 1, c.attn_head_dim, 0.f, 0.1f);
  }
}

// Rows of each tensor held by rank r of n (row sharding; outputs are
// all-gathered so every row's dot product is the 1-GPU one).
void shard_layer(const si_model& m, LayerLayout* L) {
  const si_model_config& c = m.c;
  const uint64_t H = c.hidden, I = c.intermediate, d = c.gdn_head_dim, hd = c.attn_head_dim;
  const uint64_t n = uint64_t(m.n), r = uint64_t(m.r);
  for (int id = 0; id < SI_T_COUNT; ++id) {
    LocalTensor& t = L->t[id];
    if (!t.present) continue;
    auto one = [&](uint64_t b, uint64_t e) { t.ranges = {{b, e}}; };
    switch (id) {
      case SI_T_FFN_GATE:
      case SI_T_FFN_UP: one(r * I / n, (r + 1) * I / n); break;
      case SI_T_FFN_DOWN:
      case SI_T_SSM_OUT:
      case SI_T_ATTN_O: one(r * H / n, (r + 1) * H / n); break;
      case SI_T_OUTPUT: one(r * c.vocab / n, (r + 1) * c.vocab / n); break;
      case SI_T_SSM_QKV:
      case SI_T_SSM_CONV: {
        const uint64_t kw = uint64_t(c.gdn_key_heads) * d;
        const uint64_t q0 = r * m.kh_l * d, v0 = r * m.vh_l * d;
        t.ranges = {{q0, q0 + m.kh_l * d}, {kw + q0, kw + q0 + m.kh_l * d}, {2 * kw + v0, 2 * kw + v0 + m.vh_l * d}};
        break;
      }
      case SI_T_SSM_Z: one(r * m.vh_l * d, (r + 1) * m.vh_l * d); break;
      case SI_T_SSM_ALPHA:
      case SI_T_SSM_BETA:
      case SI_T_SSM_A:
      case SI_T_SSM_DT: one(r * m.vh_l, (r + 1) * m.vh_l); break;
      case SI_T_ATTN_Q: {
        const uint64_t qw = uint64_t(c.attn_q_heads) * hd, q0 = r * m.qh_l * hd;
        t.ranges = {{q0, q0 + m.qh_l * hd}, {qw + q0, qw + q0 + m.qh_l * hd}};
        break;
      }
      case SI_T_ATTN_K:
      case SI_T_ATTN_V: one(uint64_t(m.kv_lo) * hd, uint64_t(m.kv_lo + m.kvh_l) * hd); break;
      default: one(0, t.full_rows); break;
    }
    t.rows = 0;
    for (auto& rr : t.ranges) t.rows += rr.end - rr.begin;
  }
  uint64_t off = 0;
  for (int id = 0; id < SI_T_COUNT; ++id) {
    LocalTensor& t = L->t[id];
    if (!t.present) continue;
    t.offset = off;
    t.bytes = t.rows * row_bytes_of(t.type, t.cols);
    off = align256(off + t.bytes + 64);
  }
  L->bytes = off;
}

// Generate local tensor `t` of (layer, id) into dst.
void generate_tensor(uint64_t seed, uint32_t layer, uint32_t id, const LocalTensor& t, uint8_t* dst,
                     bool centered) {
  const uint64_t key = tensor_key(seed, layer, id);
  const uint64_t rb = row_bytes_of(t.type, t.cols);
  uint8_t* p = dst;
  for (const RowRange& rr : t.ranges) {
    for (uint64_t row = rr.begin; row < rr.end; ++row) {
      if (t.type == SI_GGML_TYPE_F32) {
        float* f = reinterpret_cast<float*>(p);
        for (uint64_t cidx = 0; cidx < t.cols; ++cidx)
          f[cidx] = float(double(t.mean) + double(t.stdev) * gauss(key, row * t.cols + cidx));
      } else {
        fill_bytes(key, row * rb, rb, p);
        const uint32_t bb = block_bytes_of(t.type);
        const uint64_t bpr = t.cols / 256;
        for (uint64_t b = 0; b < bpr; ++b) {
          patch_scales(key, t.type, row * bpr + b, p + b * bb);
          if (centered && t.type != SI_GGML_TYPE_Q6_K) center_scales(key, t.type, row * bpr + b, p + b * bb);
        }
      }
      p += rb;
    }
  }
}

template <typename F>
void parallel_for(uint64_t n, F f) {
  unsigned nt = std::max(1u, std::min(64u, std::thread::hardware_concurrency()));
  std::vector<std::thread> th;
  std::atomic<uint64_t> next{0};
  for (unsigned i = 0; i < nt; ++i)
    th.emplace_back([&] {
      for (uint64_t k = next++; k < n; k = next++) f(k);
    });
  for (auto& t : th) t.join();
}

int validate_config(const si_model_config& c, int n) {
  const uint64_t nn = uint64_t(n);
  if (c.hidden == 0 || c.hidden % 256 || c.intermediate == 0 || c.intermediate % 256 ||
      c.layers == 0 || c.vocab == 0 || c.attn_interval == 0)
    return 1;
  if (c.gdn_head_dim != 128 || c.gdn_key_heads == 0 || c.gdn_value_heads % c.gdn_key_heads ||
      (uint64_t(c.gdn_value_heads) * 128) % 256 || c.conv_kernel < 2 || c.conv_kernel > 8)
    return 2;
  if (c.attn_kv_heads == 0 || c.attn_q_heads % c.attn_kv_heads || c.attn_head_dim > 256 ||
      c.attn_head_dim % 32 || c.attn_q_heads / c.attn_kv_heads > 8 ||
      (uint64_t(c.attn_q_heads) * c.attn_head_dim) % 256 || c.rotary_dim > c.attn_head_dim ||
      c.rotary_dim % 2 || c.kv_capacity == 0 || c.kv_capacity + 1 > kAttnMaxTokens)
    return 3;
  if (!(c.rms_eps > 0.f) || !std::isfinite(c.rms_eps)) return 4;
  if (block_bytes_of(c.mlp_type) == 0 || block_bytes_of(c.down_type) == 0 || block_bytes_of(c.head_type) == 0)
    return 5;
  if (c.hidden % nn || c.intermediate % nn || c.vocab % nn || c.gdn_key_heads % nn ||
      c.gdn_value_heads % nn || c.attn_q_heads % nn)
    return 6;
  const uint32_t group = c.attn_q_heads / c.attn_kv_heads, qh_l = c.attn_q_heads / n;
  if (group % qh_l && qh_l % group) return 7;
  return 0;
}


// Shard dimensions and the packed per-layer layout of rank r of n (no CUDA).
void init_shape(si_model* m) {
  const si_model_config& c = m->c;
  const int n = m->n, r = m->r;
  m->kh_l = c.gdn_key_heads / n;
  m->vh_l = c.gdn_value_heads / n;
  m->qh_l = c.attn_q_heads / n;
  const uint32_t group = c.attn_q_heads / c.attn_kv_heads;
  m->kv_lo = (uint32_t(r) * m->qh_l) / group;
  m->kvh_l = ((uint32_t(r) + 1) * m->qh_l - 1) / group + 1 - m->kv_lo;
  m->H_l = c.hidden / n;
  m->I_l = c.intermediate / n;
  m->V_l = c.vocab / n;

  // ---- layout + pinned host weights -------------------------------------
  m->layout.resize(c.layers + 1);
  for (uint32_t l = 0; l <= c.layers; ++l) {
    LayerLayout& L = m->layout[l];
    const bool globals = l == c.layers;
    L.gdn = !globals && ((l + 1) % c.attn_interval != 0);
    full_spec(c, L.gdn, globals, &L);
    if (!m->ttype.empty())
      for (int id = 0; id < SI_T_COUNT; ++id)
        if (L.t[id].present) L.t[id].type = m->ttype[l][id];
    shard_layer(*m, &L);
  }
}

// Device scratch vectors of the decode loop, in float counts.
std::vector<uint64_t> scratch_float_counts(const si_model& m) {
  const si_model_config& c = m.c;
  const uint64_t H = c.hidden, proj_l = (2ull * m.kh_l + m.vh_l) * 128;
  const uint64_t qw = uint64_t(c.attn_q_heads) * c.attn_head_dim, vw = uint64_t(c.gdn_value_heads) * 128;
  const uint64_t part_floats = attn_scratch_floats(m.qh_l, m.kvh_l, c.attn_head_dim, c.kv_capacity + 1, 256);
  return {H, H, proj_l, uint64_t(m.vh_l) * 128, 2ull * m.vh_l, uint64_t(m.vh_l) * 128, vw, vw,
          2ull * m.qh_l * c.attn_head_dim, uint64_t(m.kvh_l) * c.attn_head_dim,
          uint64_t(m.kvh_l) * c.attn_head_dim, uint64_t(m.qh_l) * c.attn_head_dim, qw, qw,
          uint64_t(m.qh_l) * c.attn_head_dim, m.I_l, c.intermediate, m.V_l, c.vocab,
          c.rotary_dim / 2 + 1, part_floats, H, m.I_l};
}

// Candidate-major buffers of the batched verifier, in float counts (b_hid,
// b_xn, b_xg, b_qkv, b_z, b_ab, b_core, b_qg, b_kk, b_vv, b_att, b_act, b_up,
// b_logits), then 8-byte argmax keys and two u32 arrays.
std::vector<uint64_t> batch_float_counts(const si_model& m) {
  const si_model_config& c = m.c;
  if (m.n != 1) return {};
  const uint64_t K = kQmmMaxBatch, H = c.hidden, d = c.gdn_head_dim;
  const uint64_t proj = (2ull * c.gdn_key_heads + c.gdn_value_heads) * d, vw = uint64_t(c.gdn_value_heads) * d;
  const uint64_t qw = uint64_t(c.attn_q_heads) * c.attn_head_dim, kvw = uint64_t(c.attn_kv_heads) * c.attn_head_dim;
  return {K * H, K * H, K * std::max(vw, qw), K * proj, K * vw, K * 2 * c.gdn_value_heads, K * vw,
          K * 2 * qw, K * kvw, K * kvw, K * qw, K * c.intermediate, K * c.intermediate, K * c.vocab};
}

// Largest tensor-core batched-matvec scratch over the model's matrices.
uint64_t batch_qmm_bytes(const si_model& m) {
  const si_model_config& c = m.c;
  const uint32_t H = c.hidden, d = c.gdn_head_dim, K = kQmmMaxBatch;
  const uint32_t proj = (2 * c.gdn_key_heads + c.gdn_value_heads) * d, vw = c.gdn_value_heads * d;
  const uint32_t qw = c.attn_q_heads * c.attn_head_dim, kvw = c.attn_kv_heads * c.attn_head_dim;
  const uint32_t shapes[][2] = {{proj, H}, {vw, H}, {2 * qw, H}, {kvw, H}, {c.intermediate, H},
                                {H, c.intermediate}, {H, vw}, {H, qw}, {c.vocab, H}};
  uint64_t b = 0;
  for (const auto& s : shapes) b = std::max(b, qmm_tc_scratch_bytes(s[0], s[1], K, 148));
  return b;
}

// The exchange area of a sharded model (n > 1; it takes the place of the
// verifier's buffers, which only one GPU has): ticket and epoch words, then
// 8-byte exchange words for two parity halves of the hidden, the activation,
// the GDN core and z, and the attention output and gate vectors.
uint64_t xchg_bytes(const si_model& m) {
  if (m.n == 1) return 0;
  const uint64_t vw = uint64_t(m.c.gdn_value_heads) * 128, qw = uint64_t(m.c.attn_q_heads) * m.c.attn_head_dim;
  return 256 + 512 + align256(16ull * m.c.hidden) + align256(16ull * m.c.intermediate) + 2 * align256(16 * vw) +
         2 * align256(16 * qw);
}

uint64_t batch_bytes(const si_model& m) {
  const std::vector<uint64_t> f = batch_float_counts(m);
  if (f.empty()) return 0;
  uint64_t b = 256;  // alignment slack after the peer flags
  for (uint64_t v : f) b += align256(v * 4);
  return b + 3 * 256 + align256(batch_qmm_bytes(m));  // keys, ids, tokens, matvec scratch
}

// The C struct of a retention policy as the context keeps it (NULL: none).
int retention_from(const si_retention* r, Retention* out, std::string* err) {
  *out = Retention{};
  if (!r) return SI_OK;
  if (r->n_layers && !r->layers) {
    *err = "retention policy lists layers without an array";
    return SI_E_INVALID;
  }
  if (r->flags & ~(SI_RETAIN_EXACT | SI_RETAIN_TENSORS)) {
    *err = "unknown retention flags " + std::to_string(r->flags);
    return SI_E_INVALID;
  }
  out->set = true;
  out->prefix = r->prefix_layers;
  out->stride = r->stride;
  out->offset = r->offset;
  out->flags = r->flags;
  out->layers.assign(r->layers, r->layers + r->n_layers);
  if (r->flags & SI_RETAIN_TENSORS) {
    out->mlp_layers = r->mlp_layers;
    out->mlp_stride = r->mlp_stride;
    out->mlp_offset = r->mlp_offset;
    out->q6_layers = r->q6_layers;
    out->down_stride = r->down_stride;
    out->down_offset = r->down_offset;
    out->attention_stride = r->attention_stride;
    out->attention_offset = r->attention_offset;
  }
  return SI_OK;
}

bool retains_stride_layer(uint32_t layer, uint32_t stride, uint32_t offset) {
  return stride != 0 && layer % stride == offset % stride;  // qwen35_runtime.rs:2270-2272
}

// The tensors of layer l that a tensor-level policy keeps resident
// (qwen35_runtime.rs:1646-1682), as a bit mask of tensor ids. The reference
// applies these forms only when no layers are retained by count (1565).
uint32_t tensor_selection(const si_model& m, const Retention* ret, uint32_t l) {
  if (!ret || !ret->set || ret->prefix != 0) return 0;
  const LayerLayout& L = m.layout[l];
  uint32_t mask = 0;
  auto add = [&](int id) {
    if (L.t[id].present) mask |= 1u << id;
  };
  if (l < ret->mlp_layers || retains_stride_layer(l, ret->mlp_stride, ret->mlp_offset)) {
    add(SI_T_FFN_GATE);
    add(SI_T_FFN_UP);
  }
  if (l < ret->q6_layers)
    for (int id = 0; id < SI_T_COUNT; ++id)
      if (L.t[id].present && L.t[id].type == SI_GGML_TYPE_Q6_K) add(id);
  if (retains_stride_layer(l, ret->down_stride, ret->down_offset)) add(SI_T_FFN_DOWN);
  if (!L.gdn && retains_stride_layer(l, ret->attention_stride, ret->attention_offset)) {
    add(SI_T_ATTN_Q);
    add(SI_T_ATTN_K);
    add(SI_T_ATTN_V);
    add(SI_T_ATTN_O);
  }
  return mask;
}

// Packs the selected tensors of a layer first (each tensor still spans
// align256(bytes + 64), so the layer's size does not change) and returns the
// bytes they occupy: the part that stays resident when the layer streams.
uint64_t pack_selected_first(LayerLayout* L, uint32_t mask) {
  uint64_t off = 0, part = 0;
  for (int pass = 0; pass < 2; ++pass) {  // pass 0: the selected tensors, pass 1: the others
    for (int id = 0; id < SI_T_COUNT; ++id) {
      LocalTensor& t = L->t[id];
      if (!t.present || (((mask >> id) & 1u) != 0) != (pass == 0)) continue;
      t.offset = off;
      off = align256(off + t.bytes + 64);
    }
    if (pass == 0) part = off;
  }
  return part;
}

// Residency plan inside `budget` (0 = unbounded): the output head and as many
// leading layers as fit stay resident (the reference's retained prefix,
// qwen35_runtime.rs:1640-1642); the rest stream through `depth` ring slots of
// the largest layer. A retention policy (si_ctx_set_retention) names layers
// that must stay resident first; with SI_RETAIN_EXACT nothing else does. Like
// plan_sequential_layers (planner.rs:174-251) a plan whose fixed part exceeds
// the budget is rejected. Pure host code.
int compute_plan(si_model* m, uint64_t budget, uint32_t depth, const Retention* ret, std::vector<bool>* res_out,
                 uint64_t* max_layer_out, std::string* err) {
  const si_model_config& c = m->c;
  m->depth = depth ? std::min(depth, 4u) : 3u;
  const uint64_t proj_l = (2ull * m->kh_l + m->vh_l) * 128;
  uint64_t state_bytes = 0;
  for (uint32_t l = 0; l < c.layers; ++l) {
    if (m->layout[l].gdn)
      state_bytes += align256(2 * proj_l * (c.conv_kernel - 1) * 4) + align256(uint64_t(m->vh_l) * 128 * 128 * 4);
    else
      state_bytes += 2 * align256(uint64_t(m->kvh_l) * c.kv_capacity * c.attn_head_dim * 2);
  }
  uint64_t scratch_bytes = 4 * 256 + 64 * kP2PMaxRanks;  // token, argmax keys, peer flags
  for (uint64_t f : scratch_float_counts(*m)) scratch_bytes += align256(f * 4);
  scratch_bytes += batch_bytes(*m) + xchg_bytes(*m);
  uint64_t max_layer = 0, all_layers = 0;
  for (uint32_t l = 0; l < c.layers; ++l) {
    max_layer = std::max(max_layer, m->layout[l].bytes);
    all_layers += m->layout[l].bytes;
  }
  const uint64_t globals_bytes = m->layout[c.layers].bytes;
  // the policy's layers (retained_layers, retains_stride_layer, the explicit
  // set; qwen35_runtime.rs:1552-1733, 2270-2280)
  std::vector<bool> want(c.layers, false);
  const bool policy = ret && ret->set, exact = policy && (ret->flags & SI_RETAIN_EXACT);
  uint64_t want_bytes = 0;
  uint32_t n_want = 0;
  if (policy) {
    for (uint32_t l : ret->layers)
      if (l >= c.layers) {
        *err = "retained layer " + std::to_string(l) + " is outside the model's " + std::to_string(c.layers) +
               " layers";
        return SI_E_INVALID;
      }
    for (uint32_t l = 0; l < c.layers; ++l)
      want[l] = l < ret->prefix || (ret->stride && l % ret->stride == ret->offset % ret->stride);
    for (uint32_t l : ret->layers) want[l] = true;
    for (uint32_t l = 0; l < c.layers; ++l)
      if (want[l]) {
        want_bytes += m->layout[l].bytes;
        n_want++;
      }
  }
  // the tensor-level parts of the layers not retained whole: their selected
  // tensors are packed first and stay resident if the layer streams
  std::vector<uint64_t> part(c.layers, 0);
  uint64_t parts_total = 0;
  for (uint32_t l = 0; l < c.layers; ++l) {
    part[l] = pack_selected_first(&m->layout[l], want[l] ? 0u : tensor_selection(*m, ret, l));
    parts_total += part[l];
  }
  uint64_t resident = globals_bytes;
  std::vector<bool> res(c.layers, false);
  bool ring = false;
  const uint64_t whole = globals_bytes + all_layers + state_bytes + scratch_bytes;
  if ((!exact && (budget == 0 || whole <= budget)) || (exact && n_want == c.layers)) {
    if (budget != 0 && whole > budget) {
      *err = "HBM budget " + std::to_string(budget) + " B cannot hold the retained layers, the output head, " +
             "state and scratch (" + std::to_string(whole) + " B)";
      return SI_E_BUDGET;
    }
    std::fill(res.begin(), res.end(), true);
    resident += all_layers;
  } else {
    ring = true;
    const uint64_t fixed = globals_bytes + m->depth * max_layer + state_bytes + scratch_bytes;
    if (budget != 0 && fixed > budget) {
      *err = "HBM budget " + std::to_string(budget) + " B cannot hold the output head, " +
             std::to_string(m->depth) + " staging slots of " + std::to_string(max_layer) +
             " B, state and scratch (" + std::to_string(fixed) + " B)";
      return SI_E_BUDGET;
    }
    uint64_t left = budget == 0 ? UINT64_MAX : budget - fixed;
    if (want_bytes + parts_total > left) {
      *err = "HBM budget " + std::to_string(budget) + " B leaves " + std::to_string(left) +
             " B beside the output head, ring, state and scratch, but the " + std::to_string(n_want) +
             " retained layers need " + std::to_string(want_bytes) + " B and the retained tensors of the others " +
             std::to_string(parts_total) + " B";
      return SI_E_BUDGET;
    }
    left -= want_bytes + parts_total;
    for (uint32_t l = 0; l < c.layers; ++l)
      if (want[l]) {
        res[l] = true;
        resident += m->layout[l].bytes;
      }
    if (!exact) {
      for (uint32_t l = 0; l < c.layers; ++l) {
        if (res[l]) continue;
        const uint64_t cost = m->layout[l].bytes - part[l];  // its part is already set aside
        if (cost > left) break;
        res[l] = true;
        left -= cost;
        resident += m->layout[l].bytes;
      }
    }
  }
  m->part_bytes.assign(c.layers, 0);
  for (uint32_t l = 0; l < c.layers; ++l)
    if (!res[l]) {
      m->part_bytes[l] = part[l];
      resident += part[l];
    }
  m->plan = si_plan_info{};
  m->plan.budget_bytes = budget;
  m->plan.resident_weight_bytes = resident;
  m->plan.ring_bytes = ring ? m->depth * max_layer : 0;
  m->plan.state_bytes = state_bytes;
  m->plan.scratch_bytes = scratch_bytes;
  m->plan.stage_depth = ring ? m->depth : 0;
  m->plan.head_resident = 1;
  m->streamed.clear();
  for (uint32_t l = 0; l < c.layers; ++l) {
    if (res[l]) {
      m->plan.resident_layers++;
    } else {
      m->plan.streamed_layers++;
      m->plan.streamed_bytes_per_token += m->layout[l].bytes - m->part_bytes[l];
      m->streamed.push_back(l);
    }
  }
  *res_out = res;
  *max_layer_out = max_layer;
  return SI_OK;
}

}  // namespace

extern "C" void si_model_config_qwen36_27b(si_model_config* c) {
  if (!c) return;
  std::memset(c, 0, sizeof(*c));
  c->hidden = 5120;
  c->intermediate = 17408;
  c->layers = 64;
  c->vocab = 248320;
  c->attn_interval = 4;
  c->attn_q_heads = 24;
  c->attn_kv_heads = 4;
  c->attn_head_dim = 256;
  c->rotary_dim = 64;
  c->rope_theta = 1.0e7f;
  c->gdn_key_heads = 16;
  c->gdn_value_heads = 48;
  c->gdn_head_dim = 128;
  c->conv_kernel = 4;
  c->rms_eps = 1.0e-6f;
  c->kv_capacity = 144;
  c->eos_token = 0xFFFFFFFFu;
  c->mlp_type = SI_GGML_TYPE_Q4_K;
  c->down_type = SI_GGML_TYPE_Q6_K;
  c->head_type = SI_GGML_TYPE_Q6_K;
  c->weight_init = 1;
}

namespace {

void free_model(si_model* m) {
  if (!m) return;
  cudaSetDevice(m->ctx->device);
  cudaDeviceSynchronize();
  for (auto* h : m->host)
    if (h) cudaFreeHost(h);
  if (m->embd_host) cudaFreeHost(m->embd_host);
  if (m->dev_resident) cudaFree(m->dev_resident);
  for (int i = 0; i < 4; ++i) {
    if (m->slot[i]) cudaFree(m->slot[i]);
    if (m->copy_done[i]) cudaEventDestroy(m->copy_done[i]);
    if (m->compute_done[i]) cudaEventDestroy(m->compute_done[i]);
  }
  if (m->state_block) cudaFree(m->state_block);
  if (m->p2p) comm_p2p_unmap(m->ctx, m->peer_block);
  if (m->scratch_block) cudaFree(m->scratch_block);
  for (cudaEvent_t e : m->tr_pool) cudaEventDestroy(e);
  if (m->tr_base) cudaEventDestroy(m->tr_base);
  if (m->accounted) {
    note_alloc(m->ctx, -int64_t(m->plan.resident_weight_bytes + m->plan.ring_bytes + m->plan.state_bytes +
                                m->plan.scratch_bytes));
    note_weights(m->ctx, -int64_t(m->plan.resident_weight_bytes));
  }
  delete m;
}

}  // namespace

namespace {

// Writes the local rows `part.ranges` of tensor (layer, id) to dst; returns
// SI_OK or an SI_E_* status with *err filled. Called from several threads.
using FillFn = std::function<int(uint32_t layer, uint32_t id, const LocalTensor& part, uint8_t* dst,
                                 std::string* err)>;

// Plan, fill the pinned host shards with `fill`, upload the resident set and
// set up state, scratch and the staging ring (shared by the synthetic and the
// GGUF-file constructors).
int create_model(si_ctx* ctx, const si_model_config* cfg, uint64_t seed,
                 std::vector<std::array<uint32_t, SI_T_COUNT>> types, const FillFn& fill, si_model** out) {
  *out = nullptr;
  const int n = ctx->nranks, r = ctx->rank;
  if (int v = validate_config(*cfg, n))
    return fail(ctx, SI_E_INVALID, "model config is invalid (check " + std::to_string(v) + ")");
  cudaSetDevice(ctx->device);
  auto* m = new si_model();
  m->ctx = ctx;
  m->c = *cfg;
  m->seed = seed;
  m->n = n;
  m->r = r;
  m->ttype = std::move(types);
  const si_model_config& c = m->c;
  init_shape(m);
  // ---- residency plan, before any allocation -----------------------------
  std::vector<bool> res;
  uint64_t max_layer = 0;
  {
    std::string perr;
    if (int prc = compute_plan(m, ctx->cfg.hbm_budget_bytes, ctx->cfg.stage_depth, &ctx->retention, &res,
                               &max_layer, &perr)) {
      free_model(m);
      return fail(ctx, prc, perr);
    }
  }
  const uint64_t resident = m->plan.resident_weight_bytes, state_bytes = m->plan.state_bytes,
                 scratch_bytes = m->plan.scratch_bytes;
  const bool ring = !m->streamed.empty();
  const std::vector<uint64_t> scratch_floats = scratch_float_counts(*m);
  const uint64_t proj_l = (2ull * m->kh_l + m->vh_l) * 128;
  m->host.assign(c.layers + 1, nullptr);
  for (uint32_t l = 0; l <= c.layers; ++l) {
    cudaError_t e = fault_fire(SI_FAULT_PINNED_ALLOC)
                        ? cudaErrorMemoryAllocation
                        : cudaHostAlloc(reinterpret_cast<void**>(&m->host[l]), m->layout[l].bytes, cudaHostAllocDefault);
    if (e != cudaSuccess) {
      m->host[l] = nullptr;
      int rc = cuda_fail(ctx, e, "pinned host allocation for model weights");
      free_model(m);
      return rc;
    }
  }
  // token_embd shard: vocab rows [r*V/n, (r+1)*V/n), mapped for zero-copy row reads
  LocalTensor embd;
  embd.present = true;
  embd.type = SI_GGML_TYPE_Q4_K;
  embd.full_rows = c.vocab;
  embd.cols = c.hidden;
  embd.ranges = {{uint64_t(r) * c.vocab / n, uint64_t(r + 1) * c.vocab / n}};
  embd.rows = m->V_l;
  const uint64_t embd_bytes = embd.rows * row_bytes_of(embd.type, embd.cols);
  {
    cudaError_t e = fault_fire(SI_FAULT_PINNED_ALLOC)
                        ? cudaErrorMemoryAllocation
                        : cudaHostAlloc(reinterpret_cast<void**>(&m->embd_host), embd_bytes + 64, cudaHostAllocMapped);
    if (e != cudaSuccess) m->embd_host = nullptr;
    if (e == cudaSuccess) e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&m->embd_dev), m->embd_host, 0);
    if (e != cudaSuccess) {
      int rc = cuda_fail(ctx, e, "mapped host allocation for token embeddings");
      free_model(m);
      return rc;
    }
  }
  // generate in parallel over (layer, tensor, row-chunk) work items
  struct Work {
    uint32_t layer, id;
    uint64_t range_idx, row0, row1;
    uint8_t* dst;
  };
  std::vector<Work> work;
  auto add_work = [&](uint32_t layer, uint32_t id, const LocalTensor& t, uint8_t* base) {
    const uint64_t rb = row_bytes_of(t.type, t.cols);
    uint64_t local = 0;
    for (uint64_t ri = 0; ri < t.ranges.size(); ++ri) {
      const RowRange& rr = t.ranges[ri];
      const uint64_t step = std::max<uint64_t>(1, (8ull << 20) / std::max<uint64_t>(rb, 1));
      for (uint64_t a = rr.begin; a < rr.end; a += step) {
        const uint64_t b = std::min(rr.end, a + step);
        work.push_back({layer, id, ri, a, b, base + (local + (a - rr.begin)) * rb});
      }
      local += rr.end - rr.begin;
    }
  };
  for (uint32_t l = 0; l <= c.layers; ++l)
    for (int id = 0; id < SI_T_COUNT; ++id)
      if (m->layout[l].t[id].present) add_work(l, uint32_t(id), m->layout[l].t[id], m->host[l] + m->layout[l].t[id].offset);
  add_work(c.layers, SI_T_TOKEN_EMBD, embd, m->embd_host);
  std::atomic<bool> fill_failed{false};
  std::mutex fill_mu;
  std::string fill_err;
  int fill_rc = SI_OK;
  parallel_for(work.size(), [&](uint64_t k) {
    if (fill_failed.load(std::memory_order_relaxed)) return;
    const Work& w = work[k];
    const LocalTensor& t = (w.id == SI_T_TOKEN_EMBD) ? embd : m->layout[w.layer].t[w.id];
    LocalTensor part = t;
    part.ranges = {{w.row0, w.row1}};
    std::string e;
    if (int frc = fill(w.layer, w.id, part, w.dst, &e)) {
      std::lock_guard<std::mutex> lk(fill_mu);
      if (!fill_failed.exchange(true)) {
        fill_rc = frc;
        fill_err = e;
      }
    }
  });
  if (fill_failed.load()) {
    free_model(m);
    return fail(ctx, fill_rc, fill_err);
  }

  // ---- device allocations -----------------------------------------------
  auto dmalloc = [&](void** p, uint64_t bytes, const char* what) -> int {
    cudaError_t e = fault_fire(SI_FAULT_DEVICE_ALLOC) ? cudaErrorMemoryAllocation : cudaMalloc(p, bytes ? bytes : 256);
    if (e != cudaSuccess) {
      *p = nullptr;
      return cuda_fail(ctx, e, what);
    }
    return SI_OK;
  };
  int rc = dmalloc(reinterpret_cast<void**>(&m->dev_resident), resident, "resident weight allocation");
  if (rc) {
    free_model(m);
    return rc;
  }
  m->dev_layer.assign(c.layers + 1, nullptr);
  {
    uint64_t off = 0;
    m->dev_part.assign(c.layers, nullptr);
    for (uint32_t l = 0; l <= c.layers; ++l) {
      if (l < c.layers && !res[l]) {
        // a streamed layer's retained tensors (packed first)
        const uint64_t pb = m->part_bytes[l];
        if (pb == 0) continue;
        m->dev_part[l] = m->dev_resident + off;
        cudaMemcpyAsync(m->dev_part[l], m->host[l], pb, cudaMemcpyHostToDevice, ctx->copy_stream);
        off += pb;
        continue;
      }
      m->dev_layer[l] = m->dev_resident + off;
      cudaMemcpyAsync(m->dev_layer[l], m->host[l], m->layout[l].bytes, cudaMemcpyHostToDevice, ctx->copy_stream);
      off += m->layout[l].bytes;
    }
  }
  if (ring) {
    for (uint32_t i = 0; i < m->depth; ++i) {
      if ((rc = dmalloc(reinterpret_cast<void**>(&m->slot[i]), max_layer, "staging ring slot"))) {
        free_model(m);
        return rc;
      }
      cudaEventCreateWithFlags(&m->copy_done[i], cudaEventDisableTiming);
      cudaEventCreateWithFlags(&m->compute_done[i], cudaEventDisableTiming);
    }
  }
  if ((rc = dmalloc(reinterpret_cast<void**>(&m->state_block), state_bytes, "state allocation")) ||
      (rc = dmalloc(reinterpret_cast<void**>(&m->scratch_block), scratch_bytes, "scratch allocation"))) {
    free_model(m);
    return rc;
  }
  cudaMemsetAsync(m->state_block, 0, state_bytes, ctx->copy_stream);
  cudaMemsetAsync(m->scratch_block, 0, scratch_bytes, ctx->copy_stream);
  {
    uint8_t* p = m->state_block;
    m->conv[0].assign(c.layers, nullptr);
    m->conv[1].assign(c.layers, nullptr);
    m->rec.assign(c.layers, nullptr);
    m->kc.assign(c.layers, nullptr);
    m->vc.assign(c.layers, nullptr);
    m->cached.assign(c.layers, 0);
    m->conv_parity.assign(c.layers, 0);
    for (uint32_t l = 0; l < c.layers; ++l) {
      if (m->layout[l].gdn) {
        const uint64_t cs = proj_l * (c.conv_kernel - 1) * 4;
        m->conv[0][l] = reinterpret_cast<float*>(p);
        m->conv[1][l] = reinterpret_cast<float*>(p + cs);
        p += align256(2 * cs);
        m->rec[l] = reinterpret_cast<float*>(p);
        p += align256(uint64_t(m->vh_l) * 128 * 128 * 4);
      } else {
        const uint64_t kvb = uint64_t(m->kvh_l) * c.kv_capacity * c.attn_head_dim * 2;
        m->kc[l] = reinterpret_cast<uint16_t*>(p);
        p += align256(kvb);
        m->vc[l] = reinterpret_cast<uint16_t*>(p);
        p += align256(kvb);
      }
    }
    uint8_t* s = m->scratch_block;
    float** dst[] = {&m->hidden, &m->slice, &m->qkv, &m->z, &m->ab, &m->core, &m->core_full, &m->z_full,
                     &m->qg, &m->kk, &m->vv, &m->att, &m->att_full, &m->gate_full, &m->gate_l, &m->act,
                     &m->act_full, &m->logits, &m->logits_full, &m->rope, &m->part, &m->embed, &m->up};
    for (size_t i = 0; i < sizeof(dst) / sizeof(dst[0]); ++i) {
      *dst[i] = reinterpret_cast<float*>(s);
      s += align256(scratch_floats[i] * 4);
    }
    m->d_token = reinterpret_cast<uint32_t*>(s);
    m->d_key = reinterpret_cast<unsigned long long*>(s + 256);
    m->d_keys = reinterpret_cast<unsigned long long*>(s + 512);
    m->flag_off = uint64_t(s + 1024 - m->scratch_block);
    if (m->n > 1) {
      const uint64_t x0 = align256(m->flag_off + 64 * kP2PMaxRanks);
      m->xchg_ticket_off = x0;
      m->xchg_epoch_off = x0 + 256;
      m->ll_hidden_off = x0 + 512;
      m->ll_act_off = m->ll_hidden_off + align256(16ull * c.hidden);
      m->ll_core_off = m->ll_act_off + align256(16ull * c.intermediate);
      m->ll_z_off = m->ll_core_off + align256(16ull * c.gdn_value_heads * 128);
      m->ll_att_off = m->ll_z_off + align256(16ull * c.gdn_value_heads * 128);
      m->ll_gate_off = m->ll_att_off + align256(16ull * c.attn_q_heads * c.attn_head_dim);
    }
    const std::vector<uint64_t> bf = batch_float_counts(*m);
    if (!bf.empty()) {
      uint8_t* b = m->scratch_block + align256(m->flag_off + 64 * kP2PMaxRanks);
      float** bdst[] = {&m->b_hid, &m->b_xn, &m->b_xg, &m->b_qkv, &m->b_z, &m->b_ab, &m->b_core,
                        &m->b_qg, &m->b_kk, &m->b_vv, &m->b_att, &m->b_act, &m->b_up, &m->b_logits};
      for (size_t i = 0; i < bf.size(); ++i) {
        *bdst[i] = reinterpret_cast<float*>(b);
        b += align256(bf[i] * 4);
      }
      m->b_keys = reinterpret_cast<unsigned long long*>(b);
      m->b_ids = reinterpret_cast<uint32_t*>(b + 256);
      m->b_tokens = reinterpret_cast<uint32_t*>(b + 512);
      m->b_qmm = b + 768;
      m->b_qmm_bytes = batch_qmm_bytes(*m);
    }
  }
  rope_freqs(c.rope_theta, c.rotary_dim, &m->rope_host);
  if (!m->rope_host.empty())
    cudaMemcpyAsync(m->rope, m->rope_host.data(), m->rope_host.size() * 4, cudaMemcpyHostToDevice, ctx->copy_stream);
  cudaError_t e = cudaStreamSynchronize(ctx->copy_stream);
  if (e != cudaSuccess) {
    rc = cuda_fail(ctx, e, "model upload");
    free_model(m);
    return rc;
  }
  // sharded: all-gathers go straight into the peers' scratch blocks over
  // NVLink (the zeroed flags are in place on every rank: the mapping is itself
  // a collective); NCCL when the context asks for it or mapping fails
  if (m->n > 1 && m->n <= kP2PMaxRanks && !(ctx->cfg.flags & SI_CTX_FLAG_NCCL_COLLECTIVES)) {
    if (comm_p2p_map(ctx, m->scratch_block, m->peer_block) == SI_OK)
      m->p2p = true;
    else
      ctx->err.clear();
  }
  note_alloc(ctx, int64_t(resident + m->plan.ring_bytes + state_bytes + scratch_bytes));
  note_weights(ctx, int64_t(resident));
  m->accounted = true;
  *out = m;
  return SI_OK;
}

}  // namespace

extern "C" int si_model_create_synthetic(si_ctx* ctx, const si_model_config* cfg, uint64_t seed,
                                         si_model** out) {
  if (!ctx || !cfg || !out) return fail(ctx, SI_E_INVALID, "invalid model arguments");
  const bool centered = cfg->weight_init == 1;
  return create_model(ctx, cfg, seed, {},
                      [seed, centered](uint32_t layer, uint32_t id, const LocalTensor& part, uint8_t* dst,
                                       std::string*) {
                        generate_tensor(seed, layer, id, part, dst, centered);
                        return SI_OK;
                      },
                      out);
}

namespace {

// GGUF tensor names of the decoder roles (qwen35_runtime.rs:419-446, 638-657;
// globals: token_embd / output_norm / output, 2122-2150).
const char* const kGgufNames[SI_T_COUNT] = {
    "attn_norm.weight", "post_attention_norm.weight", "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight",
    "attn_qkv.weight",  "attn_gate.weight",           "ssm_alpha.weight", "ssm_beta.weight", "ssm_conv1d.weight",
    "ssm_a",            "ssm_dt.bias",                "ssm_norm.weight", "ssm_out.weight",  "attn_q.weight",
    "attn_k.weight",    "attn_v.weight",              "attn_output.weight", "attn_q_norm.weight",
    "attn_k_norm.weight", "token_embd.weight",        "output_norm.weight", "output.weight"};

std::string gguf_name(uint32_t layer, uint32_t layers, int id) {
  if (layer == layers) return kGgufNames[id];
  return "blk." + std::to_string(layer) + "." + kGgufNames[id];
}

struct GgufCloser {
  void operator()(si_gguf* g) const { si_gguf_close(g); }
};

}  // namespace

extern "C" int si_model_create_gguf(si_ctx* ctx, const char* path, uint32_t kv_capacity, si_model** out) {
  if (!ctx || !path || !out) return fail(ctx, SI_E_INVALID, "invalid model arguments");
  *out = nullptr;
  si_gguf* raw = nullptr;
  {
    std::string err;
    if (int rc = gguf_parse(path, &raw, &err)) return fail(ctx, rc, err);
  }
  std::shared_ptr<si_gguf> g(raw, GgufCloser());
  si_model_config c;
  if (int rc = si_gguf_qwen35_config(g.get(), kv_capacity, &c)) return fail(ctx, rc, si_global_last_error());
  c.weight_init = 0;
  // every tensor of every layer: present, of the layer's kind
  // (qwen35_layer_kind, model.rs:748-783), of an executable type, with the
  // shape the config implies and a payload that covers it
  std::vector<std::array<uint32_t, SI_T_COUNT>> types(c.layers + 1);
  std::vector<std::array<uint64_t, SI_T_COUNT>> starts(c.layers + 1);
  for (uint32_t l = 0; l <= c.layers; ++l) {
    const bool globals = l == c.layers;
    bool gdn = false;
    if (!globals) {
      const std::string pre = "blk." + std::to_string(l) + ".";
      const bool has_delta = g->index.count(pre + "ssm_a") != 0;
      const bool has_attn = g->index.count(pre + "attn_q.weight") != 0;
      if (has_delta == has_attn)
        return fail(ctx, SI_E_INVALID, "Qwen3.6 layer " + std::to_string(l) + " does not have exactly one execution kind");
      const bool want_attn = (l + 1) % c.attn_interval == 0;
      if (has_attn != want_attn)
        return fail(ctx, SI_E_INVALID, "Qwen3.6 layer " + std::to_string(l) + " tensor kind " +
                                           (has_delta ? "GatedDeltaNet" : "FullAttention") +
                                           " disagrees with interval " + std::to_string(c.attn_interval));
      gdn = has_delta;
    }
    LayerLayout L;
    full_spec(c, gdn, globals, &L);
    if (globals) {  // the embedding table is held apart from the layer buffers
      L.t[SI_T_TOKEN_EMBD].present = true;
      L.t[SI_T_TOKEN_EMBD].type = SI_GGML_TYPE_Q4_K;
      L.t[SI_T_TOKEN_EMBD].full_rows = c.vocab;
      L.t[SI_T_TOKEN_EMBD].cols = c.hidden;
    }
    for (int id = 0; id < SI_T_COUNT; ++id) {
      const LocalTensor& want = L.t[id];
      if (!want.present) continue;
      const std::string name = gguf_name(l, c.layers, id);
      auto it = g->index.find(name);
      if (it == g->index.end()) return fail(ctx, SI_E_INVALID, "unknown GGUF tensor " + name);
      const GgufTensor& t = g->tensors[it->second];
      const bool f32_role = want.type == SI_GGML_TYPE_F32;
      uint64_t elems = 1;
      for (uint64_t d : t.dims) elems = (d && elems > UINT64_MAX / d) ? UINT64_MAX : elems * d;
      if (f32_role) {
        if (t.type != SI_GGML_TYPE_F32)  // f32_values (qwen35_runtime.rs:168-198)
          return fail(ctx, SI_E_UNSUPPORTED, "tensor " + name + " is not F32 (type " + std::to_string(t.type) + ")");
        if (elems != want.full_rows * want.cols)
          return fail(ctx, SI_E_INVALID, "tensor " + name + " has " + std::to_string(elems) + " F32 values; expected " +
                                             std::to_string(want.full_rows * want.cols));
      } else {
        // token_embd: q4_k_embedding_tensor; projections: any K-quant
        const bool ok = id == SI_T_TOKEN_EMBD ? t.type == SI_GGML_TYPE_Q4_K : block_bytes_of(t.type) != 0;
        if (!ok)
          return fail(ctx, SI_E_UNSUPPORTED, "tensor " + name + " has unsupported type " + std::to_string(t.type) +
                                                 (id == SI_T_TOKEN_EMBD ? " (token embeddings must be Q4_K)" : ""));
        if (t.ndim != 2 || t.dims[0] != want.cols || t.dims[1] != want.full_rows)
          return fail(ctx, SI_E_INVALID, "tensor " + name + " shape does not match the model config");
      }
      const uint64_t need = want.full_rows * row_bytes_of(t.type, want.cols);
      if (t.data_len < need)
        return fail(ctx, SI_E_INVALID, "tensor " + name + " payload is " + std::to_string(t.data_len) +
                                           " bytes; expected " + std::to_string(need));
      types[l][id] = t.type;
      starts[l][id] = t.data_start;
    }
  }
  // each rank reads only its row ranges of each tensor
  auto fill = [g, starts](uint32_t layer, uint32_t id, const LocalTensor& part, uint8_t* dst, std::string* err) {
    const uint64_t rb = row_bytes_of(part.type, part.cols);
    uint8_t* p = dst;
    for (const RowRange& rr : part.ranges) {
      const uint64_t bytes = (rr.end - rr.begin) * rb;
      if (int rc = gguf_read(g.get(), starts[layer][id] + rr.begin * rb, p, bytes, err)) return rc;
      p += bytes;
    }
    return SI_OK;
  };
  return create_model(ctx, &c, 0, std::move(types), fill, out);
}

extern "C" void si_model_destroy(si_model* m) { free_model(m); }

extern "C" int si_model_plan_dry(const si_model_config* cfg, int nranks, int rank, uint64_t budget,
                                 uint32_t depth, si_plan_info* out) {
  return si_model_plan_dry_retained(cfg, nranks, rank, budget, depth, nullptr, out, nullptr);
}

extern "C" int si_model_plan_dry_retained(const si_model_config* cfg, int nranks, int rank, uint64_t budget,
                                          uint32_t depth, const si_retention* r, si_plan_info* out,
                                          uint8_t* resident) {
  if (!cfg || !out || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(nullptr, SI_E_INVALID, "invalid plan arguments");
  if (int v = validate_config(*cfg, nranks))
    return fail(nullptr, SI_E_INVALID, "model config is invalid (check " + std::to_string(v) + ")");
  si_model m;
  m.c = *cfg;
  m.n = nranks;
  m.r = rank;
  init_shape(&m);
  std::vector<bool> res;
  uint64_t max_layer = 0;
  std::string err;
  Retention ret;
  if (int rc = retention_from(r, &ret, &err)) return fail(nullptr, rc, err);
  if (int rc = compute_plan(&m, budget, depth, &ret, &res, &max_layer, &err)) return fail(nullptr, rc, err);
  *out = m.plan;
  if (resident)
    for (uint32_t l = 0; l < cfg->layers; ++l) resident[l] = res[l] ? 1 : 0;
  return SI_OK;
}

extern "C" int si_model_resident_layers(const si_model* m, uint8_t* resident, uint32_t layers) {
  if (!m || !resident) return SI_E_INVALID;
  if (layers != m->c.layers) return fail(m->ctx, SI_E_INVALID, "resident-layer query needs one flag per layer");
  for (uint32_t l = 0; l < layers; ++l) resident[l] = m->dev_layer[l] ? 1 : 0;
  return SI_OK;
}

extern "C" int si_model_resident_part_bytes(const si_model* m, uint64_t* part_bytes, uint32_t layers) {
  if (!m || !part_bytes) return SI_E_INVALID;
  if (layers != m->c.layers) return fail(m->ctx, SI_E_INVALID, "resident-part query needs one value per layer");
  for (uint32_t l = 0; l < layers; ++l) part_bytes[l] = m->dev_part.empty() || !m->dev_part[l] ? 0 : m->part_bytes[l];
  return SI_OK;
}

extern "C" int si_ctx_set_retention(si_ctx* ctx, const si_retention* r) {
  if (!ctx) return SI_E_INVALID;
  Retention ret;
  std::string err;
  if (int rc = retention_from(r, &ret, &err)) return fail(ctx, rc, err);
  ctx->retention = std::move(ret);
  return SI_OK;
}

extern "C" int si_model_shard_rows(const si_model_config* cfg, int nranks, int rank, uint32_t layer,
                                   uint32_t tensor, uint64_t* ranges, uint32_t max_ranges,
                                   uint32_t* n_ranges) {
  if (!cfg || !n_ranges || nranks < 1 || rank < 0 || rank >= nranks || layer > cfg->layers ||
      tensor >= SI_T_COUNT)
    return fail(nullptr, SI_E_INVALID, "invalid shard query");
  if (int v = validate_config(*cfg, nranks))
    return fail(nullptr, SI_E_INVALID, "model config is invalid (check " + std::to_string(v) + ")");
  si_model m;
  m.c = *cfg;
  m.n = nranks;
  m.r = rank;
  init_shape(&m);
  *n_ranges = 0;
  if (tensor == SI_T_TOKEN_EMBD) {
    if (layer != cfg->layers) return SI_OK;
    if (max_ranges < 1) return fail(nullptr, SI_E_INVALID, "range buffer too small");
    ranges[0] = uint64_t(rank) * cfg->vocab / nranks;
    ranges[1] = uint64_t(rank + 1) * cfg->vocab / nranks;
    *n_ranges = 1;
    return SI_OK;
  }
  const LocalTensor& t = m.layout[layer].t[tensor];
  if (!t.present) return SI_OK;
  if (t.ranges.size() > max_ranges) return fail(nullptr, SI_E_INVALID, "range buffer too small");
  for (size_t i = 0; i < t.ranges.size(); ++i) {
    ranges[2 * i] = t.ranges[i].begin;
    ranges[2 * i + 1] = t.ranges[i].end;
  }
  *n_ranges = uint32_t(t.ranges.size());
  return SI_OK;
}

extern "C" int si_model_plan(const si_model* m, si_plan_info* out) {
  if (!m || !out) return SI_E_INVALID;
  *out = m->plan;
  return SI_OK;
}

extern "C" int si_model_host_tensor(const si_model* m, uint32_t layer, uint32_t tensor,
                                    const void** ptr, uint64_t* bytes, uint32_t* type) {
  if (!m || layer > m->c.layers || tensor >= SI_T_COUNT) return SI_E_INVALID;
  if (tensor == SI_T_TOKEN_EMBD && layer == m->c.layers) {
    if (ptr) *ptr = m->embd_host;
    if (bytes) *bytes = uint64_t(m->V_l) * row_bytes_of(SI_GGML_TYPE_Q4_K, m->c.hidden);
    if (type) *type = SI_GGML_TYPE_Q4_K;
    return SI_OK;
  }
  const LocalTensor& t = m->layout[layer].t[tensor];
  if (!t.present) {
    if (ptr) *ptr = nullptr;
    if (bytes) *bytes = 0;
    if (type) *type = 0;
    return SI_OK;
  }
  if (ptr) *ptr = m->host[layer] + t.offset;
  if (bytes) *bytes = t.bytes;
  if (type) *type = t.type;
  return SI_OK;
}

extern "C" int si_model_reset(si_model* m) {
  if (!m) return SI_E_INVALID;
  cudaSetDevice(m->ctx->device);
  cudaMemsetAsync(m->state_block, 0, m->plan.state_bytes, m->ctx->stream);
  std::fill(m->cached.begin(), m->cached.end(), 0u);
  std::fill(m->conv_parity.begin(), m->conv_parity.end(), 0u);
  return sync_and_check(m->ctx, "model reset");
}

// Qwen35Runtime::snapshot_states / restore_states (qwen35_runtime.rs:1764-1775):
// the whole state block (conv and recurrent states, KV caches) copied device
// to device on the context's stream, with the per-layer token counts and conv
// parities kept on the host. The weights, the ring and the verifier's hidden
// states are not part of it, as in the reference.
struct si_model_snapshot {
  si_ctx* ctx = nullptr;
  uint8_t* block = nullptr;
  uint64_t bytes = 0;
  std::vector<uint32_t> cached, conv_parity;
};

extern "C" int si_model_snapshot_states(si_model* m, si_model_snapshot** out) {
  if (!m || !out) return SI_E_INVALID;
  *out = nullptr;
  si_ctx* ctx = m->ctx;
  cudaSetDevice(ctx->device);
  auto* s = new si_model_snapshot();
  s->ctx = ctx;
  s->bytes = m->plan.state_bytes;
  s->cached = m->cached;
  s->conv_parity = m->conv_parity;
  cudaError_t e = fault_fire(SI_FAULT_DEVICE_ALLOC)
                      ? cudaErrorMemoryAllocation
                      : cudaMalloc(reinterpret_cast<void**>(&s->block), s->bytes ? s->bytes : 256);
  if (e != cudaSuccess) {
    s->block = nullptr;
    delete s;
    return cuda_fail(ctx, e, "state snapshot allocation");
  }
  note_alloc(ctx, int64_t(s->bytes));
  e = cudaMemcpyAsync(s->block, m->state_block, s->bytes, cudaMemcpyDeviceToDevice, ctx->stream);
  const int rc = e != cudaSuccess ? cuda_fail(ctx, e, "state snapshot copy") : sync_and_check(ctx, "state snapshot");
  if (rc) {
    si_model_snapshot_free(s);
    return rc;
  }
  *out = s;
  return SI_OK;
}

extern "C" int si_model_restore_states(si_model* m, const si_model_snapshot* s) {
  if (!m || !s) return SI_E_INVALID;
  si_ctx* ctx = m->ctx;
  if (s->ctx != ctx || s->bytes != m->plan.state_bytes || s->cached.size() != m->cached.size())
    return fail(ctx, SI_E_INVALID, "Qwen3.6 state snapshot depth does not match runtime");
  cudaSetDevice(ctx->device);
  cudaError_t e = cudaMemcpyAsync(m->state_block, s->block, s->bytes, cudaMemcpyDeviceToDevice, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "state restore copy");
  m->cached = s->cached;
  m->conv_parity = s->conv_parity;
  return sync_and_check(ctx, "state restore");
}

extern "C" void si_model_snapshot_free(si_model_snapshot* s) {
  if (!s) return;
  if (s->block) {
    cudaSetDevice(s->ctx->device);
    cudaFree(s->block);
    note_alloc(s->ctx, -int64_t(s->bytes));
  }
  delete s;
}

namespace {

// ---- staging ring ------------------------------------------------------------
// Occurrence j of the streamed-layer sequence (wrapping across tokens) uses
// slot j % depth. Copies run on the context's copy stream: occurrence j+depth
// is issued right after occurrence j's compute has been enqueued, gated by
// that compute's completion event.
// A timing event from the trace pool (recorded on a stream by the caller).
cudaEvent_t trace_event(si_model* m) {
  if (m->tr_used == m->tr_pool.size()) {
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    m->tr_pool.push_back(e);
  }
  return m->tr_pool[m->tr_used++];
}

void issue_copy(si_model* m, uint64_t occ) {
  const uint32_t s = uint32_t(occ % m->depth);
  const uint32_t l = m->streamed[occ % m->streamed.size()];
  cudaStreamWaitEvent(m->ctx->copy_stream, m->compute_done[s], 0);
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (m->tracing) {
    e0 = trace_event(m);
    e1 = trace_event(m);
    cudaEventRecord(e0, m->ctx->copy_stream);
    // the copy overwrites the slot: its previous occupant is evicted here
    if (m->slot_layer[s] >= 0)
      m->tr_recs.push_back({SI_ACT_EVICT, m->slot_layer[s], int(s), e0, e0, m->layout[m->slot_layer[s]].bytes});
  }
  // the layer's retained part stays where it is: only [part, bytes) travels
  const uint64_t pb = m->part_bytes[l];
  cudaMemcpyAsync(m->slot[s] + pb, m->host[l] + pb, m->layout[l].bytes - pb, cudaMemcpyHostToDevice,
                  m->ctx->copy_stream);
  cudaEventRecord(m->copy_done[s], m->ctx->copy_stream);
  if (m->tracing) {
    cudaEventRecord(e1, m->ctx->copy_stream);
    m->tr_recs.push_back({SI_ACT_PREFETCH, int(l), int(s), e0, e1, m->layout[l].bytes - pb});
  }
  m->slot_layer[s] = int(l);
}

// Execution of layer `l` (or the head, l == layers) bracketed by events on
// the compute stream when tracing, and always by an NVTX range named like the
// trace's operation ("layer-N", "output") for profilers; the range covers the
// host-side enqueue of the layer's work.
struct TraceScope {
  si_model* m;
  int layer, slot;
  cudaEvent_t e0 = nullptr;
  TraceScope(si_model* mm, int l, int s) : m(mm), layer(l), slot(s) {
    char name[32];
    if (l == int(m->c.layers))
      std::snprintf(name, sizeof(name), "output");
    else
      std::snprintf(name, sizeof(name), "layer-%d", l);
    nvtxRangePushA(name);
    if (m->tracing) {
      e0 = trace_event(m);
      cudaEventRecord(e0, m->ctx->stream);
    }
  }
  ~TraceScope() {
    nvtxRangePop();
    if (!e0) return;
    cudaEvent_t e1 = trace_event(m);
    cudaEventRecord(e1, m->ctx->stream);
    m->tr_recs.push_back({SI_ACT_EXECUTE, layer, slot, e0, e1, m->layout[layer].bytes});
  }
};

void ring_prime(si_model* m) {
  while (m->occ_issued < m->occ_next + m->depth) issue_copy(m, m->occ_issued++);
}

// The device address of a tensor of a layer whose packed bytes are at `base`
// (its resident copy or its ring slot); a streamed layer's retained tensors
// (below part_bytes) are at dev_part instead.
const uint8_t* tensor_ptr(const si_model* m, const uint8_t* base, uint32_t layer, int id) {
  const uint64_t off = m->layout[layer].t[id].offset;
  if (layer < m->part_bytes.size() && off < m->part_bytes[layer] && m->dev_part[layer]) return m->dev_part[layer] + off;
  return base + off;
}

QmvParams qmv_base(si_model* m, uint32_t type, uint32_t cols) {
  QmvParams p = {};
  p.type = type;
  p.cols = cols;
  p.nseg = 1;
  p.err = m->ctx->d_err;
  si::qscratch_for(m->ctx, m->ctx->stream, &p.scratch, &p.scratch_bytes);
  p.eps = m->c.rms_eps;
  return p;
}

int run_qmv(si_model* m, const QmvParams& p) {
  std::string msg;
  int rc = launch_qmv(p, m->ctx->stream, m->ctx->sm_count, true, &msg);
  return rc ? fail(m->ctx, rc, msg) : SI_OK;
}

uint32_t type_of(const si_model* m, uint32_t layer, int id) { return m->layout[layer].t[id].type; }

// A grouped matvec whose segments share x: one launch when every segment has
// the same type, else one launch per segment (a GGUF file may mix K-quants
// within a layer).
int run_group(si_model* m, QmvParams p, const uint32_t* types) {
  bool same = true;
  for (uint32_t i = 1; i < p.nseg; ++i) same = same && types[i] == types[0];
  if (same) {
    p.type = types[0];
    return run_qmv(m, p);
  }
  for (uint32_t i = 0; i < p.nseg; ++i) {
    QmvParams q = p;
    q.nseg = 1;
    q.seg[0] = p.seg[i];
    q.items = p.seg[i].rows;
    q.type = types[i];
    if (int rc = run_qmv(m, q)) return rc;
  }
  return SI_OK;
}

// Row-sharded output with residual: rows [H_l*r, H_l*(r+1)) of hidden are
// updated; with n > 1 they are written to `slice` and all-gathered.
// All-gather of one or two row-sharded vectors into their full copies (which
// live in the scratch block): NVLink peer stores when mapped, else NCCL.
int gather(si_model* m, const float* s1, float* r1, uint32_t n1, const float* s2 = nullptr, float* r2 = nullptr,
           uint32_t n2 = 0) {
  if (!m->p2p)
    return n2 ? comm_allgather2(m->ctx, s1, r1, n1, s2, r2, n2, m->ctx->stream)
              : comm_allgather(m->ctx, s1, r1, n1, m->ctx->stream);
  P2PGather g = {};
  for (int i = 0; i < m->n; ++i) g.block[i] = static_cast<uint8_t*>(m->peer_block[i]);
  g.send[0] = s1;
  g.send[1] = s2;
  g.recv_off[0] = uint64_t(reinterpret_cast<uint8_t*>(r1) - m->scratch_block);
  g.recv_off[1] = r2 ? uint64_t(reinterpret_cast<uint8_t*>(r2) - m->scratch_block) : 0;
  g.count[0] = n1;
  g.count[1] = n2;
  g.n = uint32_t(m->n);
  g.rank = uint32_t(m->r);
  g.epoch = ++m->p2p_epoch;
  g.flag_off = m->flag_off;
  g.err = m->ctx->d_err;
  launch_p2p_allgather(g, m->ctx->stream);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SI_OK : cuda_fail(m->ctx, e, "peer all-gather launch");
}

// A Q4_K or Q6_K matvec (or Q4_K SwiGLU pair) of this rank's rows whose epilogue gathers
// the whole vector into `full` on every rank over NVLink (PeerOut): no
// stand-alone all-gather launch. `ll_off` locates the vector's exchange words
// in every rank's scratch block. SI_E_UNSUPPORTED (nothing launched) when the
// peer mapping is absent or the tensor-core kernel does not take the call.
int exchange_qmv(si_model* m, QmvParams p, float* full, uint64_t ll_off, uint32_t full_len) {
  if (!m->p2p || m->n < 2 || m->n > kPeerMax) return SI_E_UNSUPPORTED;
  p.peer.n = uint32_t(m->n);
  p.peer.rank = uint32_t(m->r);
  for (int i = 0; i < m->n; ++i)
    p.peer.ll[i] = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(m->peer_block[i]) + ll_off);
  p.peer.parity_stride = full_len;
  p.peer.y = full;
  p.peer.row0 = uint32_t(m->r) * p.seg[0].rows;
  p.peer.total = uint32_t(m->n) * p.seg[0].rows;
  p.peer.ticket = reinterpret_cast<uint32_t*>(m->scratch_block + m->xchg_ticket_off);
  p.peer.epoch = reinterpret_cast<uint32_t*>(m->scratch_block + m->xchg_epoch_off);
  p.peer.wait_cycles = kWaitCycles;
  // only where one GPU would run the whole matrix on the tensor-core kernel
  // too (the kernel is chosen by the full shape, not the shard)
  QmvParams whole = p;
  whole.peer = PeerOut{};
  for (uint32_t i = 0; i < whole.nseg; ++i) whole.seg[i].rows = full_len;
  if (p.peer.total != full_len) return SI_E_UNSUPPORTED;
  const bool q6 = p.type == SI_GGML_TYPE_Q6_K;
  if (q6 ? !(qmv_tc6_eligible(whole) && qmv_tc6_eligible(p)) : !(qmv_tc_eligible(whole) && qmv_tc_supported(p)))
    return SI_E_UNSUPPORTED;
  std::string msg;
  const int rc = q6 ? launch_qmv_tc6(p, m->ctx->stream, m->ctx->sm_count, true, &msg)
                    : launch_qmv_tc(p, m->ctx->stream, m->ctx->sm_count, true, &msg);
  if (rc == SI_E_UNSUPPORTED) return rc;
  return rc ? fail(m->ctx, rc, msg) : SI_OK;
}

// The exchange of one gathered vector of the sharded model (PeerOut): its
// words at `ll_off` in every rank's scratch block, this rank's `local` rows
// at rank * local of the `total`-row vector `full`.
PeerOut xchg_out(si_model* m, uint64_t ll_off, float* full, uint32_t local, uint32_t total) {
  PeerOut po = {};
  po.n = uint32_t(m->n);
  po.rank = uint32_t(m->r);
  for (int i = 0; i < m->n; ++i)
    po.ll[i] = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(m->peer_block[i]) + ll_off);
  po.parity_stride = total;
  po.y = full;
  po.row0 = uint32_t(m->r) * local;
  po.total = total;
  po.ticket = reinterpret_cast<uint32_t*>(m->scratch_block + m->xchg_ticket_off);
  po.epoch = reinterpret_cast<uint32_t*>(m->scratch_block + m->xchg_epoch_off);
  po.wait_cycles = kWaitCycles;
  return po;
}

// Whether the sharded model's kernels gather their outputs themselves.
bool in_kernel_gathers(const si_model* m) { return m->n > 1 && m->p2p && m->n <= kPeerMax; }

int residual_matvec(si_model* m, QmvParams p, const uint8_t* w) {
  const uint32_t r0 = m->H_l * uint32_t(m->r);
  p.seg[0] = {w, m->n > 1 ? m->slice : m->hidden + r0, m->hidden + r0, m->H_l, 0};
  p.items = m->H_l;
  if (m->n > 1) {
    // the residual rows are read by the CTA that owns them before their new
    // value leaves, so the gather may write `hidden` in place
    const int xrc = exchange_qmv(m, p, m->hidden, m->ll_hidden_off, m->c.hidden);
    if (xrc != SI_E_UNSUPPORTED) return xrc;
  }
  int rc = run_qmv(m, p);
  if (rc) return rc;
  if (m->n > 1) return gather(m, m->slice, m->hidden, m->H_l);
  return SI_OK;
}

int mlp(si_model* m, uint32_t l, const uint8_t* base) {
  const si_model_config& c = m->c;
  const uint32_t tg = type_of(m, l, SI_T_FFN_GATE), tu = type_of(m, l, SI_T_FFN_UP);
  QmvParams p = qmv_base(m, tg, c.hidden);
  p.nseg = 2;
  p.pair = 1;
  p.seg[0] = {tensor_ptr(m, base, l, SI_T_FFN_GATE), m->act, nullptr, m->I_l, 0};
  p.seg[1] = {tensor_ptr(m, base, l, SI_T_FFN_UP), m->act, nullptr, m->I_l, 0};
  p.items = m->I_l;
  p.xmode = XM_RMS1P;
  p.x = m->hidden;
  p.xw = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_POST_NORM));
  int rc;
  const float* act = m->act;
  bool gathered = false;
  if (tg == tu && m->n > 1) {
    rc = exchange_qmv(m, p, m->act_full, m->ll_act_off, c.intermediate);
    gathered = rc == SI_OK;
    if (rc != SI_E_UNSUPPORTED && rc != SI_OK) return rc;
    if (gathered) act = m->act_full;
  }
  if (gathered) {
    rc = SI_OK;
  } else if (tg == tu) {
    rc = run_qmv(m, p);  // fused SwiGLU pair
  } else {
    p.pair = 0;
    p.seg[1].y = m->up;
    const uint32_t types[2] = {tg, tu};
    rc = run_group(m, p, types);
    if (!rc) launch_swiglu(m->act, m->up, m->act, m->I_l, m->ctx->stream);
  }
  if (rc) return rc;
  if (m->n > 1 && !gathered) {
    if ((rc = gather(m, m->act, m->act_full, m->I_l))) return rc;
    act = m->act_full;
  }
  QmvParams d = qmv_base(m, type_of(m, l, SI_T_FFN_DOWN), c.intermediate);
  d.x = act;
  d.xmode = XM_RAW;
  return residual_matvec(m, d, tensor_ptr(m, base, l, SI_T_FFN_DOWN));
}

int gdn_layer(si_model* m, uint32_t l, const uint8_t* base) {
  const si_model_config& c = m->c;
  const uint32_t proj_l = (2 * m->kh_l + m->vh_l) * 128, vw_l = m->vh_l * 128;
  const float* attn_norm = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_ATTN_NORM));
  QmvParams p = qmv_base(m, SI_GGML_TYPE_Q4_K, c.hidden);
  p.nseg = 2;
  p.seg[0] = {tensor_ptr(m, base, l, SI_T_SSM_QKV), m->qkv, nullptr, proj_l, 0};
  p.seg[1] = {tensor_ptr(m, base, l, SI_T_SSM_Z), m->z, nullptr, vw_l, 0};
  p.items = proj_l + vw_l;
  p.xmode = XM_RMS1P;
  p.x = m->hidden;
  p.xw = attn_norm;
  const uint32_t types[2] = {type_of(m, l, SI_T_SSM_QKV), type_of(m, l, SI_T_SSM_Z)};
  int rc = run_group(m, p, types);
  if (rc) return rc;
  GdnLayerArgs g = {};
  // alpha and beta (F32 rows) are projected inside the GDN step kernel
  g.alpha_w = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_ALPHA));
  g.beta_w = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_BETA));
  g.ab_x = m->hidden;
  g.ab_norm = attn_norm;
  g.ab_cols = c.hidden;
  g.ab_eps = c.rms_eps;
  g.qkv = m->qkv;
  g.conv_w = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_CONV));
  const uint32_t par = m->conv_parity[l];
  g.conv_in = m->conv[par][l];
  g.conv_out = m->conv[par ^ 1][l];
  g.state = m->rec[l];
  g.a_log = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_A));
  g.dt_bias = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_DT));
  g.core = m->core;
  g.key_heads = m->kh_l;
  g.value_heads = m->vh_l;
  g.kernel = c.conv_kernel;
  g.err = m->ctx->d_err;
  // sharded over NVLink peers: core and z are gathered inside the GDN kernel
  const bool xg = in_kernel_gathers(m);
  if (xg) {
    const uint32_t vw = c.gdn_value_heads * 128;
    g.xcore = xchg_out(m, m->ll_core_off, m->core_full, vw_l, vw);
    g.xz = xchg_out(m, m->ll_z_off, m->z_full, vw_l, vw);
    g.z_in = m->z;
  }
  launch_gdn_layer(g, m->ctx->stream, true);
  m->conv_parity[l] = par ^ 1;
  const float* core = m->core;
  const float* z = m->z;
  if (m->n > 1) {
    if (!xg && (rc = gather(m, m->core, m->core_full, vw_l, m->z, m->z_full, vw_l))) return rc;
    core = m->core_full;
    z = m->z_full;
  }
  QmvParams o = qmv_base(m, type_of(m, l, SI_T_SSM_OUT), c.gdn_value_heads * 128);
  o.xmode = XM_GATED;
  o.x = core;
  o.xaux = z;
  o.xw = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_NORM));
  o.head_dim = 128;
  return residual_matvec(m, o, tensor_ptr(m, base, l, SI_T_SSM_OUT));
}

int attn_layer(si_model* m, uint32_t l, const uint8_t* base, uint64_t position) {
  const si_model_config& c = m->c;
  const uint32_t hd = c.attn_head_dim, qw_l = m->qh_l * hd, kvw_l = m->kvh_l * hd;
  if (m->cached[l] >= c.kv_capacity) return fail(m->ctx, SI_E_STATE, "full-attention KV cache capacity exhausted");
  QmvParams p = qmv_base(m, SI_GGML_TYPE_Q4_K, c.hidden);
  p.nseg = 3;
  p.seg[0] = {tensor_ptr(m, base, l, SI_T_ATTN_Q), m->qg, nullptr, 2 * qw_l, 0};
  p.seg[1] = {tensor_ptr(m, base, l, SI_T_ATTN_K), m->kk, nullptr, kvw_l, 0};
  p.seg[2] = {tensor_ptr(m, base, l, SI_T_ATTN_V), m->vv, nullptr, kvw_l, 0};
  p.items = 2 * qw_l + 2 * kvw_l;
  p.xmode = XM_RMS1P;
  p.x = m->hidden;
  p.xw = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_ATTN_NORM));
  const uint32_t types[3] = {type_of(m, l, SI_T_ATTN_Q), type_of(m, l, SI_T_ATTN_K), type_of(m, l, SI_T_ATTN_V)};
  int rc = run_group(m, p, types);
  if (rc) return rc;
  AttnArgs a = {};
  a.q = m->qg;
  a.k_new = m->kk;
  a.v_new = m->vv;
  a.k_cache = m->kc[l];
  a.v_cache = m->vc[l];
  a.k_cache_w = m->kc[l];
  a.v_cache_w = m->vc[l];
  a.q_norm = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_ATTN_QNORM));
  a.k_norm = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_ATTN_KNORM));
  a.rope_freq = c.rotary_dim ? m->rope : nullptr;
  a.position = uint32_t(position);
  a.cached = m->cached[l];
  a.qh = m->qh_l;
  a.kvh = m->kvh_l;
  a.hd = hd;
  a.cap = c.kv_capacity;
  a.rotary = c.rotary_dim;
  a.eps = c.rms_eps;
  a.cache_bf16 = 1;
  a.part = m->part;
  a.out = m->att;
  a.chunk = 256;
  a.err = m->ctx->d_err;
  // sharded over NVLink peers: output and gate are gathered inside the merge
  const bool xg = in_kernel_gathers(m);
  if (xg) {
    const uint32_t qw = c.attn_q_heads * hd;
    a.xatt = xchg_out(m, m->ll_att_off, m->att_full, qw_l, qw);
    a.xgate = xchg_out(m, m->ll_gate_off, m->gate_full, qw_l, qw);
    a.gate_in = m->qg + qw_l;  // the gate half of the local q projection
  }
  launch_attention(a, m->ctx->stream, true);
  m->cached[l]++;
  const float* att = m->att;
  const float* gate = m->qg + qw_l;
  if (m->n > 1) {
    // gate half of the local q projection is contiguous after the queries
    if (!xg && (rc = gather(m, m->att, m->att_full, qw_l, m->qg + qw_l, m->gate_full, qw_l)))
      return rc;
    att = m->att_full;
    gate = m->gate_full;
  }
  QmvParams o = qmv_base(m, type_of(m, l, SI_T_ATTN_O), c.attn_q_heads * hd);
  o.xmode = XM_SIGGATE;
  o.x = att;
  o.xaux = gate;
  return residual_matvec(m, o, tensor_ptr(m, base, l, SI_T_ATTN_O));
}

// The layer loop over resident layers and the staging ring; `body` runs one
// layer from its device copy.
template <typename F>
int run_layers(si_model* m, F body) {
  const si_model_config& c = m->c;
  const bool ring = !m->streamed.empty();
  if (ring) ring_prime(m);
  for (uint32_t l = 0; l < c.layers; ++l) {
    const uint8_t* base = m->dev_layer[l];
    uint32_t s = 0;
    if (!base) {
      s = uint32_t(m->occ_next % m->depth);
      cudaStreamWaitEvent(m->ctx->stream, m->copy_done[s], 0);
      base = m->slot[s];
    }
    int rc;
    {
      TraceScope ts(m, int(l), m->dev_layer[l] ? -1 : int(s));
      rc = body(l, base);
    }
    if (rc) return rc;
    if (!m->dev_layer[l]) {
      cudaEventRecord(m->compute_done[s], m->ctx->stream);
      m->occ_next++;
      issue_copy(m, m->occ_issued++);
    }
  }
  return SI_OK;
}

// decode_hidden on device buffers: m->hidden is updated in place.
int decode_layers(si_model* m, uint64_t position) {
  return run_layers(m, [&](uint32_t l, const uint8_t* base) {
    int rc = m->layout[l].gdn ? gdn_layer(m, l, base) : attn_layer(m, l, base, position);
    return rc ? rc : mlp(m, l, base);
  });
}

int embed_dev(si_model* m) {
  const uint32_t lo = m->V_l * uint32_t(m->r);
  launch_embed(m->embd_dev, m->c.hidden, m->d_token, lo, lo + m->V_l, m->hidden, m->ctx->stream);
  if (m->n > 1) return comm_allreduce_sum(m->ctx, m->hidden, m->hidden, m->c.hidden, m->ctx->stream);
  return SI_OK;
}

// logits slice + global argmax into d_token (and optionally full logits).
int head_dev(si_model* m, bool gather_logits) {
  const si_model_config& c = m->c;
  TraceScope ts(m, int(c.layers), -1);
  const uint8_t* base = m->dev_layer[c.layers];
  QmvParams p = qmv_base(m, type_of(m, c.layers, SI_T_OUTPUT), c.hidden);
  p.seg[0] = {tensor_ptr(m, base, c.layers, SI_T_OUTPUT), m->logits, nullptr, m->V_l, 0};
  p.items = m->V_l;
  p.xmode = XM_RMS1P;
  p.x = m->hidden;
  p.xw = reinterpret_cast<const float*>(tensor_ptr(m, base, c.layers, SI_T_OUTPUT_NORM));
  int rc = run_qmv(m, p);
  if (rc) return rc;
  cudaMemsetAsync(m->d_key, 0, 8, m->ctx->stream);
  launch_argmax_key(m->logits, m->V_l, m->V_l * uint32_t(m->r), m->d_key, m->ctx->stream);
  if (m->n > 1) {
    if ((rc = comm_allgather_u64(m->ctx, m->d_key, m->d_keys, m->ctx->stream))) return rc;
    launch_argmax_finish(m->d_keys, uint32_t(m->n), m->d_token, m->ctx->stream);
    if (gather_logits && (rc = comm_allgather(m->ctx, m->logits, m->logits_full, m->V_l, m->ctx->stream)))
      return rc;
  } else {
    launch_argmax_finish(m->d_key, 1, m->d_token, m->ctx->stream);
  }
  return SI_OK;
}

int set_token(si_model* m, uint32_t token) {
  if (token >= m->c.vocab) return fail(m->ctx, SI_E_INVALID, "Q4_K embedding token id or dimension is invalid");
  cudaError_t e = cudaMemcpyAsync(m->d_token, &token, 4, cudaMemcpyHostToDevice, m->ctx->stream);
  return e == cudaSuccess ? SI_OK : cuda_fail(m->ctx, e, "token upload");
}

}  // namespace

extern "C" int si_model_embed(si_model* m, uint32_t token, float* hidden_out) {
  if (!m || !hidden_out) return SI_E_INVALID;
  cudaSetDevice(m->ctx->device);
  int rc = set_token(m, token);
  if (!rc) rc = embed_dev(m);
  if (rc) return rc;
  cudaMemcpyAsync(hidden_out, m->hidden, m->c.hidden * 4, cudaMemcpyDeviceToHost, m->ctx->stream);
  return sync_and_check(m->ctx, "embedding command");
}

extern "C" int si_model_decode_hidden(si_model* m, uint64_t position, float* hidden) {
  if (!m || !hidden) return SI_E_INVALID;
  cudaSetDevice(m->ctx->device);
  cudaMemcpyAsync(m->hidden, hidden, m->c.hidden * 4, cudaMemcpyHostToDevice, m->ctx->stream);
  int rc = decode_layers(m, position);
  if (rc) return rc;
  cudaMemcpyAsync(hidden, m->hidden, m->c.hidden * 4, cudaMemcpyDeviceToHost, m->ctx->stream);
  return sync_and_check(m->ctx, "decode_hidden");
}

extern "C" int si_model_logits(si_model* m, const float* hidden, float* logits) {
  if (!m || !hidden || !logits) return SI_E_INVALID;
  cudaSetDevice(m->ctx->device);
  cudaMemcpyAsync(m->hidden, hidden, m->c.hidden * 4, cudaMemcpyHostToDevice, m->ctx->stream);
  int rc = head_dev(m, true);
  if (rc) return rc;
  cudaMemcpyAsync(logits, m->n > 1 ? m->logits_full : m->logits, uint64_t(m->c.vocab) * 4, cudaMemcpyDeviceToHost,
                  m->ctx->stream);
  return sync_and_check(m->ctx, "logits");
}

extern "C" int si_model_decode_token(si_model* m, uint32_t token, uint64_t position, uint32_t* next,
                                     float* logits) {
  if (!m) return SI_E_INVALID;
  cudaSetDevice(m->ctx->device);
  int rc = set_token(m, token);
  if (!rc) rc = embed_dev(m);
  if (!rc) rc = decode_layers(m, position);
  if (!rc) rc = head_dev(m, logits != nullptr);
  if (rc) return rc;
  uint32_t id = 0;
  cudaMemcpyAsync(&id, m->d_token, 4, cudaMemcpyDeviceToHost, m->ctx->stream);
  if (logits)
    cudaMemcpyAsync(logits, m->n > 1 ? m->logits_full : m->logits, uint64_t(m->c.vocab) * 4,
                    cudaMemcpyDeviceToHost, m->ctx->stream);
  if ((rc = sync_and_check(m->ctx, "decode_token"))) return rc;
  if (id == 0xffffffffu) return fail(m->ctx, SI_E_INVALID, "logits contain no finite values");
  if (next) *next = id;
  return SI_OK;
}

extern "C" int si_model_generate(si_model* m, const uint32_t* prompt, uint64_t n_prompt,
                                 uint64_t max_new, uint32_t* out_ids, uint64_t* n_out) {
  if (!m || (!prompt && n_prompt) || (!out_ids && max_new) || !n_out) return SI_E_INVALID;
  if (n_prompt == 0) return fail(m->ctx, SI_E_INVALID, "prompt must contain at least one token");
  cudaSetDevice(m->ctx->device);
  *n_out = 0;
  int rc;
  // prefill, token by token (runtime.rs:3571-3576)
  for (uint64_t p = 0; p < n_prompt; ++p) {
    if ((rc = set_token(m, prompt[p])) || (rc = embed_dev(m)) || (rc = decode_layers(m, p))) return rc;
  }
  if ((rc = head_dev(m, false))) return rc;
  // greedy loop (runtime.rs:3588-3600)
  for (uint64_t i = 0; i < max_new; ++i) {
    uint32_t id = 0;
    cudaMemcpyAsync(&id, m->d_token, 4, cudaMemcpyDeviceToHost, m->ctx->stream);
    if ((rc = sync_and_check(m->ctx, "generation step"))) return rc;
    if (id == 0xffffffffu) return fail(m->ctx, SI_E_INVALID, "logits contain no finite values");
    out_ids[i] = id;
    *n_out = i + 1;
    if (id == m->c.eos_token) break;
    // the token id is already in d_token: embed it directly on the device
    if ((rc = embed_dev(m)) || (rc = decode_layers(m, n_prompt + i)) || (rc = head_dev(m, false))) return rc;
  }
  return sync_and_check(m->ctx, "generation");
}

// ---- batched verifier (qwen35_runtime.rs:879-1289, 2048-2120, 2194-2227) ----
namespace {

// One batched matvec over `batch` candidate inputs [batch][ldx]; out rows
// [batch][ldy], optionally accumulated onto resid (y may alias resid).
int run_qmm(si_model* m, uint32_t type, const uint8_t* w, uint32_t rows, uint32_t cols, uint32_t batch,
            const float* x, uint64_t ldx, float* y, uint64_t ldy, const float* resid = nullptr) {
  QmmParams p = {};
  p.type = type;
  p.rows = rows;
  p.cols = cols;
  p.batch = batch;
  p.w = w;
  p.x = x;
  p.ldx = ldx;
  p.y = y;
  p.ldy = ldy;
  p.resid = resid;
  p.ldr = ldy;
  p.scratch = m->b_qmm;
  p.scratch_bytes = m->b_qmm_bytes;
  p.err = m->ctx->d_err;
  si::qscratch_for(m->ctx, m->ctx->stream, &p.qscratch, &p.qscratch_bytes);
  std::string msg;
  int rc = launch_qmm(p, m->ctx->stream, m->ctx->sm_count, true, &msg);
  return rc ? fail(m->ctx, rc, msg) : SI_OK;
}

// GDN token mixer for a candidate window: projections batched, conv and
// recurrence candidate by candidate (each sees the previous one's state),
// gated norm batched, ssm_out batched onto the residual.
int gdn_many(si_model* m, uint32_t l, const uint8_t* base, uint32_t K) {
  const si_model_config& c = m->c;
  const uint32_t H = c.hidden, vh = c.gdn_value_heads, proj = (2 * c.gdn_key_heads + vh) * 128, vw = vh * 128;
  const float* attn_norm = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_ATTN_NORM));
  launch_rms_norm_heads(m->b_hid, attn_norm, K, H, c.rms_eps, m->b_xn, m->ctx->stream);
  int rc = run_qmm(m, type_of(m, l, SI_T_SSM_QKV), tensor_ptr(m, base, l, SI_T_SSM_QKV), proj, H, K, m->b_xn, H,
                   m->b_qkv, proj);
  if (!rc)
    rc = run_qmm(m, type_of(m, l, SI_T_SSM_Z), tensor_ptr(m, base, l, SI_T_SSM_Z), vw, H, K, m->b_xn, H, m->b_z, vw);
  if (rc) return rc;
  for (uint32_t k = 0; k < K; ++k) {
    float* ab = m->b_ab + uint64_t(k) * 2 * vh;
    launch_f32_matvec_norm2(reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_ALPHA)), ab,
                            reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_BETA)), ab + vh, vh, H,
                            m->b_hid + uint64_t(k) * H, attn_norm, c.rms_eps, m->ctx->stream);
    GdnLayerArgs g = {};
    g.qkv = m->b_qkv + uint64_t(k) * proj;
    g.conv_w = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_CONV));
    const uint32_t par = m->conv_parity[l];
    g.conv_in = m->conv[par][l];
    g.conv_out = m->conv[par ^ 1][l];
    g.state = m->rec[l];
    g.alpha = ab;
    g.beta_logit = ab + vh;
    g.a_log = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_A));
    g.dt_bias = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_DT));
    g.core = m->b_core + uint64_t(k) * vw;
    g.key_heads = c.gdn_key_heads;
    g.value_heads = vh;
    g.kernel = c.conv_kernel;
    launch_gdn_layer(g, m->ctx->stream, false);
    m->conv_parity[l] = par ^ 1;
  }
  launch_rms_norm_gated(m->b_core, m->b_z, reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_SSM_NORM)),
                        K * vh, 128, c.rms_eps, m->b_xg, m->ctx->stream);
  return run_qmm(m, type_of(m, l, SI_T_SSM_OUT), tensor_ptr(m, base, l, SI_T_SSM_OUT), H, vw, K, m->b_xg, vw,
                 m->b_hid, H, m->b_hid);
}

// Full-attention mixer for a candidate window: q/k/v batched, then per
// candidate norm + RoPE at its position, cache append and attention over the
// cache so far; gating batched; the output projection batched onto the residual.
int attn_many(si_model* m, uint32_t l, const uint8_t* base, uint32_t K, const uint64_t* positions) {
  const si_model_config& c = m->c;
  const uint32_t H = c.hidden, hd = c.attn_head_dim, qw = c.attn_q_heads * hd, kvw = c.attn_kv_heads * hd;
  launch_rms_norm_heads(m->b_hid, reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_ATTN_NORM)), K, H,
                        c.rms_eps, m->b_xn, m->ctx->stream);
  int rc = run_qmm(m, type_of(m, l, SI_T_ATTN_Q), tensor_ptr(m, base, l, SI_T_ATTN_Q), 2 * qw, H, K, m->b_xn, H,
                   m->b_qg, 2 * qw);
  if (!rc)
    rc = run_qmm(m, type_of(m, l, SI_T_ATTN_K), tensor_ptr(m, base, l, SI_T_ATTN_K), kvw, H, K, m->b_xn, H, m->b_kk,
                 kvw);
  if (!rc)
    rc = run_qmm(m, type_of(m, l, SI_T_ATTN_V), tensor_ptr(m, base, l, SI_T_ATTN_V), kvw, H, K, m->b_xn, H, m->b_vv,
                 kvw);
  if (rc) return rc;
  for (uint32_t k = 0; k < K; ++k) {
    AttnArgs a = {};
    a.q = m->b_qg + uint64_t(k) * 2 * qw;
    a.k_new = m->b_kk + uint64_t(k) * kvw;
    a.v_new = m->b_vv + uint64_t(k) * kvw;
    a.k_cache = m->kc[l];
    a.v_cache = m->vc[l];
    a.k_cache_w = m->kc[l];
    a.v_cache_w = m->vc[l];
    a.q_norm = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_ATTN_QNORM));
    a.k_norm = reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_ATTN_KNORM));
    a.rope_freq = c.rotary_dim ? m->rope : nullptr;
    a.position = uint32_t(positions[k]);
    a.cached = m->cached[l];
    a.qh = c.attn_q_heads;
    a.kvh = c.attn_kv_heads;
    a.hd = hd;
    a.cap = c.kv_capacity;
    a.rotary = c.rotary_dim;
    a.eps = c.rms_eps;
    a.cache_bf16 = 1;
    a.part = m->part;
    a.out = m->b_att + uint64_t(k) * qw;
    a.chunk = 256;
    a.err = m->ctx->d_err;
    launch_attention(a, m->ctx->stream, false);
    m->cached[l]++;
  }
  // the gate half of each candidate's q projection follows its queries
  launch_siggate_many(m->b_att, qw, m->b_qg + qw, 2 * qw, m->b_xg, qw, qw, K, m->ctx->stream);
  return run_qmm(m, type_of(m, l, SI_T_ATTN_O), tensor_ptr(m, base, l, SI_T_ATTN_O), H, qw, K, m->b_xg, qw,
                 m->b_hid, H, m->b_hid);
}

int mlp_many(si_model* m, uint32_t l, const uint8_t* base, uint32_t K) {
  const si_model_config& c = m->c;
  const uint32_t H = c.hidden, I = c.intermediate;
  launch_rms_norm_heads(m->b_hid, reinterpret_cast<const float*>(tensor_ptr(m, base, l, SI_T_POST_NORM)), K, H,
                        c.rms_eps, m->b_xn, m->ctx->stream);
  int rc = run_qmm(m, type_of(m, l, SI_T_FFN_GATE), tensor_ptr(m, base, l, SI_T_FFN_GATE), I, H, K, m->b_xn, H,
                   m->b_act, I);
  if (!rc)
    rc = run_qmm(m, type_of(m, l, SI_T_FFN_UP), tensor_ptr(m, base, l, SI_T_FFN_UP), I, H, K, m->b_xn, H, m->b_up, I);
  if (rc) return rc;
  launch_swiglu(m->b_act, m->b_up, m->b_act, uint64_t(K) * I, m->ctx->stream);
  return run_qmm(m, type_of(m, l, SI_T_FFN_DOWN), tensor_ptr(m, base, l, SI_T_FFN_DOWN), H, I, K, m->b_act, I,
                 m->b_hid, H, m->b_hid);
}

int check_batch(si_model* m, uint32_t n, const char* what) {
  if (n == 0 || n > kQmmMaxBatch)
    return fail(m->ctx, SI_E_INVALID, std::string("Qwen3.6 ") + what + " must contain 1..8 tokens");
  if (m->n != 1 || !m->b_hid)
    return fail(m->ctx, SI_E_UNSUPPORTED, "batched verification runs on an unsharded model");
  return SI_OK;
}

// Embed the window's tokens and run every layer over it (hidden states stay
// in b_hid).
int decode_many_dev(si_model* m, const uint32_t* tokens, const uint64_t* positions, uint32_t K) {
  const si_model_config& c = m->c;
  for (uint32_t k = 0; k < K; ++k)
    if (tokens[k] >= c.vocab) return fail(m->ctx, SI_E_INVALID, "token id is out of range");
  for (uint32_t l = 0; l < c.layers; ++l)
    if (!m->layout[l].gdn && m->cached[l] + K > c.kv_capacity)
      return fail(m->ctx, SI_E_STATE, "batched full-attention KV cache capacity exhausted");
  cudaMemcpyAsync(m->b_tokens, tokens, K * 4, cudaMemcpyHostToDevice, m->ctx->stream);
  for (uint32_t k = 0; k < K; ++k)
    launch_embed(m->embd_dev, c.hidden, m->b_tokens + k, 0, c.vocab, m->b_hid + uint64_t(k) * c.hidden,
                 m->ctx->stream);
  m->b_valid = 0;
  int rc = run_layers(m, [&](uint32_t l, const uint8_t* base) {
    int r = m->layout[l].gdn ? gdn_many(m, l, base, K) : attn_many(m, l, base, K, positions);
    return r ? r : mlp_many(m, l, base, K);
  });
  if (!rc) m->b_valid = K;
  return rc;
}

// Output norm, head and per-candidate argmax over b_hid.
int logits_many_dev(si_model* m, uint32_t K) {
  const si_model_config& c = m->c;
  TraceScope ts(m, int(c.layers), -1);
  const uint8_t* base = m->dev_layer[c.layers];
  launch_rms_norm_heads(m->b_hid, reinterpret_cast<const float*>(tensor_ptr(m, base, c.layers, SI_T_OUTPUT_NORM)),
                        K, c.hidden, c.rms_eps, m->b_xn, m->ctx->stream);
  int rc = run_qmm(m, type_of(m, c.layers, SI_T_OUTPUT), tensor_ptr(m, base, c.layers, SI_T_OUTPUT), c.vocab,
                   c.hidden, K, m->b_xn, c.hidden, m->b_logits, c.vocab);
  if (rc) return rc;
  cudaMemsetAsync(m->b_keys, 0, K * 8, m->ctx->stream);
  for (uint32_t k = 0; k < K; ++k) {
    launch_argmax_key(m->b_logits + uint64_t(k) * c.vocab, c.vocab, 0, m->b_keys + k, m->ctx->stream);
    launch_argmax_finish(m->b_keys + k, 1, m->b_ids + k, m->ctx->stream);
  }
  return SI_OK;
}

int read_many(si_model* m, uint32_t K, float* logits, uint32_t* ids, const char* what) {
  std::vector<uint32_t> idv(K);
  cudaMemcpyAsync(idv.data(), m->b_ids, K * 4, cudaMemcpyDeviceToHost, m->ctx->stream);
  if (logits)
    cudaMemcpyAsync(logits, m->b_logits, uint64_t(K) * m->c.vocab * 4, cudaMemcpyDeviceToHost, m->ctx->stream);
  if (int rc = sync_and_check(m->ctx, what)) return rc;
  for (uint32_t k = 0; k < K; ++k)
    if (idv[k] == 0xffffffffu) return fail(m->ctx, SI_E_INVALID, "logits contain no finite values");
  if (ids) std::memcpy(ids, idv.data(), K * 4);
  return SI_OK;
}

}  // namespace

extern "C" int si_model_decode_tokens_many(si_model* m, const uint32_t* tokens, const uint64_t* positions,
                                           uint32_t n, float* hidden_out) {
  if (!m || !tokens || !positions) return SI_E_INVALID;
  if (int rc = check_batch(m, n, "candidate window")) return rc;
  cudaSetDevice(m->ctx->device);
  if (int rc = decode_many_dev(m, tokens, positions, n)) return rc;
  if (hidden_out)
    cudaMemcpyAsync(hidden_out, m->b_hid, uint64_t(n) * m->c.hidden * 4, cudaMemcpyDeviceToHost, m->ctx->stream);
  return sync_and_check(m->ctx, "decode_tokens_many");
}

extern "C" int si_model_logits_many(si_model* m, const float* hidden, uint32_t n, float* logits, uint32_t* ids) {
  if (!m) return SI_E_INVALID;
  if (int rc = check_batch(m, n, "batched logits")) return rc;
  cudaSetDevice(m->ctx->device);
  if (hidden) {
    cudaMemcpyAsync(m->b_hid, hidden, uint64_t(n) * m->c.hidden * 4, cudaMemcpyHostToDevice, m->ctx->stream);
    m->b_valid = n;
  } else if (m->b_valid != n) {
    return fail(m->ctx, SI_E_STATE, "no device hidden states for this window: pass hidden");
  }
  if (int rc = logits_many_dev(m, n)) return rc;
  return read_many(m, n, logits, ids, "logits_many");
}

extern "C" int si_model_verify_many(si_model* m, const uint32_t* tokens, const uint64_t* positions, uint32_t n,
                                    uint32_t* ids, float* logits) {
  if (!m || !tokens || !positions) return SI_E_INVALID;
  if (int rc = check_batch(m, n, "candidate window")) return rc;
  cudaSetDevice(m->ctx->device);
  if (int rc = decode_many_dev(m, tokens, positions, n)) return rc;
  if (int rc = logits_many_dev(m, n)) return rc;
  return read_many(m, n, logits, ids, "verify_many");
}

// ---- measured planner trace -------------------------------------------------
namespace {

// A resident layer is "blk.N"; a copy staged in a ring slot is "blk.N@ring-S"
// (one layer can sit in two slots at once when fewer layers stream than the
// ring has slots).
std::string layer_tensor(const si_model* m, int l, int slot) {
  const std::string base = l == int(m->c.layers) ? std::string("output") : "blk." + std::to_string(l);
  return slot >= 0 ? base + "@ring-" + std::to_string(slot) : base;
}

std::string layer_op(const si_model* m, int l) {
  return l == int(m->c.layers) ? std::string("output") : "layer-" + std::to_string(l);
}

uint64_t process_rss() {
  FILE* f = std::fopen("/proc/self/statm", "r");
  unsigned long long size = 0, res = 0;
  if (f) {
    if (std::fscanf(f, "%llu %llu", &size, &res) != 2) res = 0;
    std::fclose(f);
  }
  return uint64_t(res) * uint64_t(sysconf(_SC_PAGESIZE));
}

}  // namespace

extern "C" int si_model_trace_begin(si_model* m) {
  if (!m) return SI_E_INVALID;
  if (m->tracing) return fail(m->ctx, SI_E_STATE, "a trace is already being recorded");
  cudaSetDevice(m->ctx->device);
  if (!m->tr_base && cudaEventCreate(&m->tr_base) != cudaSuccess)
    return fail(m->ctx, SI_E_CUDA, "trace event creation failed");
  m->tr_recs.clear();
  m->tr_used = 0;
  // time zero on the compute stream; the copy stream starts after it
  cudaEventRecord(m->tr_base, m->ctx->stream);
  cudaStreamWaitEvent(m->ctx->copy_stream, m->tr_base, 0);
  // what is in HBM when the trace starts: the resident layers and head, and
  // whatever the ring has already staged
  for (uint32_t l = 0; l <= m->c.layers; ++l)
    if (m->dev_layer[l]) m->tr_recs.push_back({SI_ACT_RETAIN, int(l), -1, nullptr, nullptr, m->layout[l].bytes});
  for (uint32_t s = 0; s < m->depth; ++s)
    if (!m->streamed.empty() && m->slot_layer[s] >= 0)
      m->tr_recs.push_back({SI_ACT_RETAIN, m->slot_layer[s], int(s), nullptr, nullptr,
                            m->layout[m->slot_layer[s]].bytes});
  m->tracing = true;
  return SI_OK;
}

extern "C" int si_model_trace_end(si_model* m, si_trace** out) {
  if (!m || !out) return SI_E_INVALID;
  *out = nullptr;
  if (!m->tracing) return fail(m->ctx, SI_E_STATE, "no trace is being recorded");
  m->tracing = false;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->copy_stream);
  if (int rc = sync_and_check(m->ctx, "trace")) return rc;
  auto ns_of = [&](cudaEvent_t e) -> uint64_t {
    if (!e) return 0;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, m->tr_base, e) != cudaSuccess || ms < 0.f) return 0;
    return uint64_t(double(ms) * 1e6);
  };
  struct Item {
    si::TraceAction a;
    size_t rec;
    int order;
  };
  std::vector<Item> items;
  items.reserve(m->tr_recs.size());
  for (size_t i = 0; i < m->tr_recs.size(); ++i) {
    const auto& r = m->tr_recs[i];
    si::TraceAction a;
    a.kind = r.kind;
    a.tier = SI_TIER_HBM;
    a.op = layer_op(m, r.layer);
    a.tensors = {layer_tensor(m, r.layer, r.slot)};
    a.bytes = r.bytes;
    a.started_ns = ns_of(r.e0);
    a.ended_ns = std::max(a.started_ns, ns_of(r.e1));
    const std::string where = r.slot >= 0 ? "ring slot " + std::to_string(r.slot) : std::string("resident");
    switch (r.kind) {
      case SI_ACT_RETAIN:
        a.queue = "transfer";
        a.reason = r.slot >= 0 ? "staged in " + where + " before the trace began" : "resident for the whole run";
        break;
      case SI_ACT_PREFETCH:
        a.queue = "transfer";
        a.reason = "stage streamed layer into " + where + " ahead of its execution";
        break;
      case SI_ACT_EVICT:
        a.queue = "transfer";
        a.reason = "overwrite " + where + " with the next streamed layer";
        break;
      default:
        a.queue = "compute";
        a.reason = "execute with its weights " + (r.slot >= 0 ? "in " + where : std::string("resident"));
    }
    // at equal start times: retained, evicted, prefetched, then executed
    const int order = r.kind == SI_ACT_RETAIN ? 0 : r.kind == SI_ACT_EVICT ? 1 : r.kind == SI_ACT_PREFETCH ? 2 : 3;
    items.push_back({std::move(a), i, order});
  }
  std::stable_sort(items.begin(), items.end(), [](const Item& x, const Item& y) {
    return x.a.started_ns != y.a.started_ns ? x.a.started_ns < y.a.started_ns : x.order < y.order;
  });
  auto* t = new si_trace();
  t->core.mode = m->streamed.empty() ? SI_MODE_RESIDENT : SI_MODE_OVERLAP;
  std::string err;
  // SI-003 invariants on the measured device times (timer resolution ~0.5 us):
  // an execution starts after its prefetch landed; an eviction starts after
  // the evicted layer's last execution ended
  constexpr float kTol = 1e-3f;  // ms
  std::map<std::pair<int, int>, cudaEvent_t> landed, done;  // (layer, slot)
  for (const Item& it : items) {
    const auto& r = m->tr_recs[it.rec];
    float ms = 0.f;
    const std::pair<int, int> key{r.layer, r.slot};
    if (r.kind == SI_ACT_PREFETCH) landed[key] = r.e1;
    if (r.kind == SI_ACT_EXECUTE) {
      if (r.slot >= 0 && landed.count(key) && landed[key] &&
          cudaEventElapsedTime(&ms, landed[key], r.e0) == cudaSuccess && ms < -kTol)
        err = "SI-003: " + layer_op(m, r.layer) + " started " + std::to_string(-ms * 1e3) +
              " us before its prefetch landed";
      done[key] = r.e1;
    }
    if (r.kind == SI_ACT_EVICT && done.count(key) &&
        cudaEventElapsedTime(&ms, done[key], r.e0) == cudaSuccess && ms < -kTol)
      err = "SI-003: " + layer_op(m, r.layer) + " was evicted " + std::to_string(-ms * 1e3) +
            " us before its execution ended";
    if (!err.empty()) break;
    if (int rc = t->core.record(it.a, &err)) {
      delete t;
      return fail(m->ctx, rc, err);
    }
  }
  if (!err.empty()) {
    delete t;
    return fail(m->ctx, SI_E_STATE, err);
  }
  t->core.observed = true;
  t->core.observed_peak_hbm = m->ctx->peak_allocated.load();
  t->core.observed_peak_rss = process_rss();
  m->tr_recs.clear();
  *out = t;
  return SI_OK;
}
