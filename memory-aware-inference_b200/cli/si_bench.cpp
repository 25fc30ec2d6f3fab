// si-bench for the CUDA backend: the reference's command line (src/main.rs:
// 1-176: flags, usage, error texts, exit codes 0 / 1 / 2) and its reports
// (src/lib.rs:45-207 RunReport and run_mock; src/runtime.rs:2689-2850
// ResidentReport, 3380-3555 run_gguf_resident / run_gguf_generation) over the
// C ABI of libsi_cuda.so.
//
// Backends: "mock" (the reference's deterministic plumbing check, no device),
// "cuda-resident" (every layer in HBM) and "cuda-streaming" (a bounded HBM
// budget with the staging ring); the reference's names "metal-resident" and
// "metal-streaming" select the same two. Models: a qwen35 GGUF file, or
// "synthetic:27b" / "synthetic:small" (seeded Qwen3.6-27B-shaped weights).
// The tokenizer is not part of this backend: CUDA runs take the prompt as
// token ids (--prompt-ids) and report the generated ids, space-separated, as
// the generated output.
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cinttypes>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <optional>
#include <sstream>
#include <string>
#include <vector>

#include "si_cuda.h"

namespace {

const char* kUsage =
    "Usage: si-bench --model PATH --backend mock|cuda-streaming|cuda-resident --prompt TEXT [options]\n\n"
    "Options:\n"
    "  --max-tokens N          Generated tokens (default: 32)\n"
    "  --context N             Maximum context capacity (default: 2048)\n"
    "  --chunk-rows N          Stream matvec weights in row chunks\n"
    "  --retain-output-head   Keep the LM head resident (always the case here)\n"
    "  --retain-layers N       Keep the first N transformer layers resident (streaming backend)\n"
    "  --quality-fixture PATH  Run the versioned capability suite (slow, opt-in)\n"
    "  --warmup N              Warmup runs (default: 1)\n"
    "  --repetitions N         Measured repetitions (default: 3)\n"
    "  --verify-manifest       Verify pinned model file digests\n"
    "  --output text|json      Report format (default: text)\n"
    "  --expected-output TEXT  Compare generated text\n"
    "  --prompt-ids LIST       Prompt as comma-separated token ids (CUDA backends)\n"
    "  --hbm-budget-gb X       HBM bound for the streaming backend (default: 4)\n"
    "  --device N              CUDA device ordinal (default: 0)\n"
    "  -h, --help              Show this help\n\n"
    "Models: a qwen35 GGUF file, synthetic:27b or synthetic:small. The metal-resident and\n"
    "metal-streaming backend names select the CUDA backends.";

struct Config {
  std::string model_path, backend, prompt;
  bool has_prompt = false;
  uint32_t max_tokens = 32;
  uint64_t max_context = 2048;
  std::optional<uint64_t> chunk_rows;
  bool retain_output_head = false;
  uint64_t retain_layers = 0;
  std::optional<std::string> quality_fixture;
  uint32_t warmup = 1, repetitions = 3;
  bool verify_manifest = false, json = false;
  std::optional<std::string> expected_output;
  std::vector<uint32_t> prompt_ids;
  bool has_prompt_ids = false;
  double hbm_budget_gb = 4.0;
  int device = 0;
};

struct ParseError {
  std::string msg;
};

// positive_u32 / positive_usize (main.rs:126-138)
uint64_t positive(const std::string& flag, const std::string& v, uint64_t max) {
  if (v.empty() || v.find_first_not_of("0123456789") != std::string::npos) throw ParseError{flag + " must be a positive integer"};
  errno = 0;
  const unsigned long long n = std::strtoull(v.c_str(), nullptr, 10);
  if (errno || n == 0 || n > max) throw ParseError{flag + " must be a positive integer"};
  return n;
}

// parse_args (main.rs:42-124); nullopt: print the usage and exit 0
std::optional<Config> parse_args(const std::vector<std::string>& args) {
  if (args.empty()) return std::nullopt;
  for (const auto& a : args)
    if (a == "--help" || a == "-h") return std::nullopt;
  Config c;
  std::optional<std::string> model, backend;
  for (size_t i = 0; i < args.size();) {
    const std::string& flag = args[i];
    if (flag == "--verify-manifest") {
      c.verify_manifest = true;
      ++i;
      continue;
    }
    if (flag == "--retain-output-head") {
      c.retain_output_head = true;
      ++i;
      continue;
    }
    if (i + 1 >= args.size()) throw ParseError{"missing value for " + flag};
    const std::string& v = args[i + 1];
    if (flag == "--model") model = v;
    else if (flag == "--backend") backend = v;
    else if (flag == "--prompt") c.prompt = v, c.has_prompt = true;
    else if (flag == "--max-tokens") c.max_tokens = uint32_t(positive(flag, v, 0xffffffffull));
    else if (flag == "--context") c.max_context = positive(flag, v, UINT64_MAX);
    else if (flag == "--chunk-rows") c.chunk_rows = positive(flag, v, UINT64_MAX);
    else if (flag == "--retain-layers") c.retain_layers = positive(flag, v, UINT64_MAX);
    else if (flag == "--quality-fixture") c.quality_fixture = v;
    else if (flag == "--warmup") {
      if (v.empty() || v.find_first_not_of("0123456789") != std::string::npos || v.size() > 9)
        throw ParseError{flag + " must be a non-negative integer"};
      c.warmup = uint32_t(std::strtoul(v.c_str(), nullptr, 10));
    } else if (flag == "--repetitions") c.repetitions = uint32_t(positive(flag, v, 0xffffffffull));
    else if (flag == "--output") {
      if (v == "text") c.json = false;
      else if (v == "json") c.json = true;
      else throw ParseError{"--output must be text or json"};
    } else if (flag == "--expected-output") c.expected_output = v;
    else if (flag == "--prompt-ids") {
      c.has_prompt_ids = true;
      std::stringstream ss(v);
      std::string tok;
      while (std::getline(ss, tok, ',')) {
        if (tok.empty() || tok.find_first_not_of("0123456789") != std::string::npos || tok.size() > 10)
          throw ParseError{"--prompt-ids must be comma-separated token ids"};
        const unsigned long long id = std::strtoull(tok.c_str(), nullptr, 10);
        if (id > 0xffffffffull) throw ParseError{"--prompt-ids must be comma-separated token ids"};
        c.prompt_ids.push_back(uint32_t(id));
      }
      if (c.prompt_ids.empty()) throw ParseError{"--prompt-ids must be comma-separated token ids"};
    } else if (flag == "--hbm-budget-gb") {
      char* end = nullptr;
      c.hbm_budget_gb = std::strtod(v.c_str(), &end);
      if (!end || *end || !(c.hbm_budget_gb > 0)) throw ParseError{"--hbm-budget-gb must be a positive number"};
    } else if (flag == "--device") {
      if (v.empty() || v.find_first_not_of("0123456789") != std::string::npos || v.size() > 4)
        throw ParseError{"--device must be a non-negative integer"};
      c.device = std::atoi(v.c_str());
    }
    else throw ParseError{"unknown option: " + flag};
    i += 2;
  }
  if (!backend) throw ParseError{"--backend is required"};
  std::string b = *backend;
  if (b == "metal-resident") b = "cuda-resident";
  if (b == "metal-streaming") b = "cuda-streaming";
  if (b != "mock" && b != "cuda-resident" && b != "cuda-streaming")
    throw ParseError{"unsupported backend: " + *backend +
                     "; available: mock, cuda-streaming, cuda-resident (metal-streaming, metal-resident)"};
  c.backend = *backend;
  if (!model) throw ParseError{"--model is required"};
  c.model_path = *model;
  if (!c.has_prompt && !c.has_prompt_ids) throw ParseError{"--prompt is required"};
  return c;
}

// json_escape (lib.rs:189-206): quotes, backslashes, \n \r \t, and other
// control characters (C0, DEL and the UTF-8 encoded C1 range) as \u00XX
std::string json_escape(const std::string& v) {
  std::string o;
  for (size_t i = 0; i < v.size(); ++i) {
    const unsigned char ch = static_cast<unsigned char>(v[i]);
    if (ch == 0xC2 && i + 1 < v.size() && (static_cast<unsigned char>(v[i + 1]) & 0xE0) == 0x80) {
      char buf[8];
      std::snprintf(buf, sizeof(buf), "\\u%04x", static_cast<unsigned char>(v[i + 1]));
      o += buf;
      ++i;
      continue;
    }
    switch (ch) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (ch < 0x20 || ch == 0x7f) {
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", ch);
          o += buf;
        } else {
          o += char(ch);
        }
    }
  }
  return o;
}

double rate(uint64_t tokens, double seconds) { return seconds <= 0 ? 0.0 : double(tokens) / seconds; }
const char* option_bool(std::optional<bool> v) { return !v ? "null" : (*v ? "true" : "false"); }

std::string fmt3(double v) {
  char b[64];
  std::snprintf(b, sizeof(b), "%.3f", v);
  return b;
}

uint32_t token_count(const std::string& t) {  // whitespace-separated words (lib.rs:170-172)
  std::stringstream ss(t);
  std::string w;
  uint32_t n = 0;
  while (ss >> w) ++n;
  return n;
}

// run_mock (lib.rs:124-168) and RunReport (lib.rs:45-121)
int run_mock(const Config& c) {
  const uint32_t prompt_tokens = token_count(c.prompt);
  std::string out;
  for (uint32_t i = 0; i < c.max_tokens; ++i) out += (i ? " mock-" : "mock-") + std::to_string(i);
  volatile uint64_t sink = 0;
  for (uint32_t i = 0; i < c.warmup; ++i) sink += token_count(c.prompt);
  auto t0 = std::chrono::steady_clock::now();
  uint64_t sum = 0;
  for (unsigned char ch : c.prompt) sum += ch;
  sink += sum;
  const double prefill = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  t0 = std::chrono::steady_clock::now();
  for (uint32_t w = token_count(out); w; --w) sink += w;
  const double decode = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  const uint64_t vram = 64 + c.max_tokens / 8, ram = 32 + c.model_path.size() / 64;
  std::optional<bool> match;
  if (c.expected_output) match = *c.expected_output == out;
  if (!c.json) {
    std::printf(
        "model=%s\nbackend=%s\nprompt_tokens=%u\ngenerated_tokens=%u\nwarmup_runs=%u\nprefill_ms=%s\ndecode_ms=%s\n"
        "prefill_tok_s=%s\ndecode_tok_s=%s\ntotal_tok_s=%s\npeak_vram_mib=%" PRIu64 "\npeak_ram_mib=%" PRIu64
        "\noutput_match=%s\ngenerated_output=%s\n",
        c.model_path.c_str(), c.backend.c_str(), prompt_tokens, c.max_tokens, c.warmup, fmt3(prefill * 1e3).c_str(),
        fmt3(decode * 1e3).c_str(), fmt3(rate(prompt_tokens, prefill)).c_str(),
        fmt3(rate(c.max_tokens, decode)).c_str(), fmt3(rate(prompt_tokens + c.max_tokens, prefill + decode)).c_str(),
        vram, ram, option_bool(match), out.c_str());
  } else {
    std::printf(
        "{\"model_path\":\"%s\",\"backend\":\"%s\",\"prompt_tokens\":%u,\"generated_tokens\":%u,\"warmup_runs\":%u,"
        "\"prefill_ms\":%s,\"decode_ms\":%s,\"prefill_tok_s\":%s,\"decode_tok_s\":%s,\"total_tok_s\":%s,"
        "\"peak_vram_mib\":%" PRIu64 ",\"peak_ram_mib\":%" PRIu64 ",\"output_match\":%s,\"generated_output\":\"%s\"}\n",
        json_escape(c.model_path).c_str(), json_escape(c.backend).c_str(), prompt_tokens, c.max_tokens, c.warmup,
        fmt3(prefill * 1e3).c_str(), fmt3(decode * 1e3).c_str(), fmt3(rate(prompt_tokens, prefill)).c_str(),
        fmt3(rate(c.max_tokens, decode)).c_str(), fmt3(rate(prompt_tokens + c.max_tokens, prefill + decode)).c_str(),
        vram, ram, option_bool(match), json_escape(out).c_str());
  }
  return match == std::optional<bool>(false) ? 2 : 0;
}

struct Failure {
  std::string msg;
};

void check(int rc, si_ctx* ctx, const char* what) {
  if (rc == SI_OK) return;
  const char* m = ctx ? si_last_error(ctx) : si_global_last_error();
  throw Failure{std::string(what) + ": " + (m && *m ? m : "failed (status " + std::to_string(rc) + ")")};
}

uint64_t rss_bytes() {  // resident set of this process (pinned host weights included)
  std::ifstream f("/proc/self/statm");
  uint64_t size = 0, res = 0;
  f >> size >> res;
  return res * uint64_t(sysconf(_SC_PAGESIZE));
}

template <typename T>
T median(std::vector<T> v) {  // median_duration / median_u64 (runtime.rs:4079-4102)
  if (v.empty()) return T();
  std::sort(v.begin(), v.end());
  return v[v.size() / 2];
}

bool is_gguf(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  char m[4] = {};
  return f.read(m, 4) && std::memcmp(m, "GGUF", 4) == 0;
}

struct Measured {
  double prefill, decode;
  uint64_t peak_vram_mib, peak_ram_mib;
  std::vector<uint32_t> ids;
};

// run_gguf_generation (runtime.rs:3557-3614): the prompt advances the state
// token by token and its last step yields the first greedy id (prefill); each
// non-EOS generated id, the last requested one included, advances it once more.
// SI_PROFILE_QWEN35 (qwen35_runtime.rs:1786, 1920-1926, 2185-2190): one line
// per layer and per output head on stderr, in the reference's format. The
// reference times each layer on the host; here the layer loop only enqueues
// work, so the times are the device's, taken from the measured trace of the
// call (CUDA events around each layer's kernels).
template <typename F>
void profiled(si_ctx* ctx, si_model* m, F call) {
  static const bool on = std::getenv("SI_PROFILE_QWEN35") != nullptr;
  if (!on) {
    call();
    return;
  }
  check(si_model_trace_begin(m), ctx, "profile trace");
  call();
  si_trace* t = nullptr;
  check(si_model_trace_end(m, &t), ctx, "profile trace");
  uint64_t n = 0;
  si_trace_count(t, &n);
  for (uint64_t i = 0; i < n; ++i) {
    si_trace_action a;
    if (si_trace_action_at(t, i, &a) != SI_OK || a.kind != SI_ACT_EXECUTE) continue;
    const double ms = double(a.ended_ns - a.started_ns) / 1e6;
    const std::string op = a.operation_id;
    if (op == "output")
      std::fprintf(stderr, "si_qwen35_output_head ms=%.3f\n", ms);
    else if (op.rfind("layer-", 0) == 0)
      std::fprintf(stderr, "si_qwen35_layer layer=%s ms=%.3f\n", op.c_str() + 6, ms);
  }
  si_trace_destroy(t);
}

Measured generate(si_ctx* ctx, si_model* m, const std::vector<uint32_t>& prompt, uint32_t max_new, uint32_t eos,
                  uint64_t hidden) {
  Measured r{};
  uint64_t peak_rss = rss_bytes();
  std::vector<float> h(hidden);
  auto t0 = std::chrono::steady_clock::now();
  for (size_t p = 0; p + 1 < prompt.size(); ++p) {
    check(si_model_embed(m, prompt[p], h.data()), ctx, "embed");
    profiled(ctx, m, [&] { check(si_model_decode_hidden(m, p, h.data()), ctx, "decode"); });
    peak_rss = std::max(peak_rss, rss_bytes());
  }
  uint32_t next = 0;
  profiled(ctx, m, [&] {
    check(si_model_decode_token(m, prompt.back(), prompt.size() - 1, &next, nullptr), ctx, "prefill");
  });
  r.prefill = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  t0 = std::chrono::steady_clock::now();
  for (uint32_t i = 0; i < max_new; ++i) {
    r.ids.push_back(next);
    if (next == eos) break;
    profiled(ctx, m, [&] {
      check(si_model_decode_token(m, next, prompt.size() + i, &next, nullptr), ctx, "decode_token");
    });
    peak_rss = std::max(peak_rss, rss_bytes());
  }
  r.decode = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  si_stats st;
  check(si_get_stats(ctx, &st), ctx, "stats");
  r.peak_vram_mib = st.peak_allocated_bytes >> 20;
  r.peak_ram_mib = peak_rss >> 20;
  return r;
}

// run_gguf_resident (runtime.rs:3380-3555) on the CUDA backend
int run_cuda(const Config& c) {
  if (c.repetitions == 0) throw Failure{"measured repetitions must be non-zero"};
  if (c.quality_fixture)
    throw Failure{"the pinned quality fixture belongs to the Qwen3-4B Safetensors model; omit --quality-fixture for the GGUF canonical run"};
  if (c.chunk_rows) throw Failure{"GGUF canonical execution does not accept --chunk-rows"};
  if (!c.has_prompt_ids)
    throw Failure{"this backend has no tokenizer: pass the prompt as token ids with --prompt-ids"};
  const bool synthetic = c.model_path.rfind("synthetic:", 0) == 0;
  struct stat sb;
  if (!synthetic) {
    if (stat(c.model_path.c_str(), &sb) != 0) throw Failure{"stat model " + c.model_path + ": " + std::strerror(errno)};
    if (S_ISDIR(sb.st_mode)) throw Failure{"BF16 Safetensors model directories are not supported by this backend"};
    if (!is_gguf(c.model_path))
      throw Failure{"unsupported model container " + c.model_path + "; expected a Safetensors directory or GGUF file"};
  }
  si_model_config mc;
  std::string revision = "qwen3.6-27b-q4-gguf";
  uint64_t mapped = 0, context_length = UINT64_MAX;
  if (synthetic) {
    si_model_config_qwen36_27b(&mc);
    if (c.model_path == "synthetic:small") {
      mc.hidden = 512, mc.intermediate = 1024, mc.layers = 8, mc.vocab = 4096, mc.attn_q_heads = 4;
      mc.attn_kv_heads = 2, mc.attn_head_dim = 128, mc.rotary_dim = 32, mc.gdn_key_heads = 2, mc.gdn_value_heads = 4;
    } else if (c.model_path != "synthetic:27b") {
      throw Failure{"unknown synthetic model " + c.model_path + "; available: synthetic:27b, synthetic:small"};
    }
    revision = "synthetic-" + c.model_path.substr(10);
    mc.kv_capacity = uint32_t(std::min<uint64_t>(c.max_context, 0xfffffffeull));
  } else {
    si_gguf* g = nullptr;
    check(si_gguf_open(c.model_path.c_str(), &g), nullptr, "open GGUF model");
    const int rc = si_gguf_qwen35_config(g, uint32_t(std::min<uint64_t>(c.max_context, 0xfffffffeull)), &mc);
    const char* name = nullptr;
    if (si_gguf_meta_string(g, "general.name", &name) == SI_OK && name) revision = name;
    uint64_t cl = 0;
    if (si_gguf_meta_u64(g, "qwen35.context_length", &cl) == SI_OK) context_length = cl;
    si_gguf_close(g);
    check(rc, nullptr, "GGUF config");
    mapped = uint64_t(sb.st_size);
  }
  if (c.retain_layers > mc.layers)
    throw Failure{"requested " + std::to_string(c.retain_layers) + " retained layers exceeds GGUF model depth " +
                  std::to_string(mc.layers)};
  if (c.max_context > context_length)
    throw Failure{"requested context " + std::to_string(c.max_context) + " exceeds GGUF model capacity " +
                  std::to_string(context_length)};
  if (c.prompt_ids.size() + c.max_tokens > c.max_context)
    throw Failure{"prompt plus generation exceeds context capacity"};
  for (uint32_t id : c.prompt_ids)
    if (id >= mc.vocab) throw Failure{"prompt token id " + std::to_string(id) + " is outside the vocabulary"};

  const bool streaming = c.backend == "cuda-streaming" || c.backend == "metal-streaming";
  si_ctx_config cc = {};
  cc.stage_depth = 3;
  // --retain-layers N: the first N layers resident and every other layer
  // streamed (new_with_retained_layers_and_head, qwen35_runtime.rs:1552);
  // otherwise the budget decides
  if (streaming && !c.retain_layers) cc.hbm_budget_bytes = uint64_t(c.hbm_budget_gb * double(1ull << 30));
  si_device_info dev;
  check(si_device_probe(c.device, &dev), nullptr, "device probe");
  si_ctx* ctx = nullptr;
  check(si_ctx_create(c.device, &cc, &ctx), nullptr, "context");
  if (streaming && c.retain_layers) {
    si_retention keep = {};
    keep.prefix_layers = uint32_t(c.retain_layers);
    keep.flags = SI_RETAIN_EXACT;
    check(si_ctx_set_retention(ctx, &keep), ctx, "retention");
  }
  si_model* m = nullptr;
  std::vector<Measured> runs;
  si_plan_info plan{};
  try {
    if (synthetic)
      check(si_model_create_synthetic(ctx, &mc, 27, &m), ctx, "model");
    else
      check(si_model_create_gguf(ctx, c.model_path.c_str(), mc.kv_capacity, &m), ctx, "model");
    check(si_model_plan(m, &plan), ctx, "plan");
    for (uint32_t w = 0; w < c.warmup; ++w) {
      check(si_model_reset(m), ctx, "reset");
      generate(ctx, m, c.prompt_ids, c.max_tokens, mc.eos_token, mc.hidden);
    }
    for (uint32_t r = 0; r < c.repetitions; ++r) {
      check(si_model_reset(m), ctx, "reset");
      check(si_reset_peaks(ctx), ctx, "reset peaks");
      runs.push_back(generate(ctx, m, c.prompt_ids, c.max_tokens, mc.eos_token, mc.hidden));
    }
  } catch (...) {
    if (m) si_model_destroy(m);
    si_ctx_destroy(ctx);
    throw;
  }
  si_stats st;
  si_get_stats(ctx, &st);
  si_model_destroy(m);
  si_ctx_destroy(ctx);

  const Measured& first = runs.front();
  bool reps_match = true;
  for (const auto& r : runs) reps_match = reps_match && r.ids == first.ids;
  std::string out, ids;
  for (size_t i = 0; i < first.ids.size(); ++i) {
    out += (i ? " " : "") + std::to_string(first.ids[i]);
    ids += (i ? "," : "") + std::to_string(first.ids[i]);
  }
  std::vector<double> pre, dec;
  std::vector<uint64_t> vram, ram;
  for (const auto& r : runs) {
    pre.push_back(r.prefill);
    dec.push_back(r.decode);
    vram.push_back(r.peak_vram_mib);
    ram.push_back(r.peak_ram_mib);
  }
  const double prefill = median(pre), decode = median(dec);
  const uint64_t pt = c.prompt_ids.size(), gt = first.ids.size();
  std::optional<bool> match;
  if (c.expected_output) match = *c.expected_output == out;
  const std::string label = "rss_plus_cuda_device; pinned_host_weights_in_rss";
  const uint64_t ws_mib = dev.total_bytes >> 20;
  const uint64_t peak_v = *std::max_element(vram.begin(), vram.end()), peak_r = *std::max_element(ram.begin(), ram.end());
  if (!c.json) {
    std::printf(
        "model=%s\nmodel_revision=%s\nbackend=%s\ndevice=%s\nprompt_tokens=%" PRIu64 "\ngenerated_tokens=%" PRIu64
        "\nwarmup_runs=%u\nrepetitions=%u\nprefill_ms=%s\ndecode_ms=%s\nprefill_tok_s=%s\ndecode_tok_s=%s\n"
        "total_tok_s=%s\nrecommended_working_set_mib=%" PRIu64 "\nmapped_model_bytes=%" PRIu64
        "\nactive_weight_bytes=%" PRIu64 "\nkv_bytes=%" PRIu64 "\nscratch_bytes=%" PRIu64 "\npeak_vram_mib=%" PRIu64
        "\npeak_ram_mib=%" PRIu64 "\nmedian_peak_vram_mib=%" PRIu64 "\nmedian_peak_ram_mib=%" PRIu64
        "\npeak_memory_aggregation=worst\nmemory_measurement=%s\noutput_match=%s\nrepetition_outputs_match=%s\n"
        "quality_present=false\ngenerated_output=%s\n",
        c.model_path.c_str(), revision.c_str(), c.backend.c_str(), dev.name, pt, gt, c.warmup, c.repetitions,
        fmt3(prefill * 1e3).c_str(), fmt3(decode * 1e3).c_str(), fmt3(rate(pt, prefill)).c_str(),
        fmt3(rate(gt, decode)).c_str(), fmt3(rate(pt + gt, prefill + decode)).c_str(), ws_mib, mapped,
        st.peak_active_weight_bytes, plan.state_bytes, plan.scratch_bytes, peak_v, peak_r, median(vram), median(ram),
        label.c_str(), option_bool(match), reps_match ? "true" : "false", out.c_str());
  } else {
    std::printf(
        "{\"model_path\":\"%s\",\"model_revision\":\"%s\",\"backend\":\"%s\",\"device\":\"%s\",\"prompt_tokens\":%" PRIu64
        ",\"generated_tokens\":%" PRIu64 ",\"warmup_runs\":%u,\"repetitions\":%u,\"prefill_ms\":%s,\"decode_ms\":%s,"
        "\"prefill_tok_s\":%s,\"decode_tok_s\":%s,\"total_tok_s\":%s,\"recommended_working_set_mib\":%" PRIu64
        ",\"mapped_model_bytes\":%" PRIu64 ",\"active_weight_bytes\":%" PRIu64 ",\"kv_bytes\":%" PRIu64
        ",\"scratch_bytes\":%" PRIu64 ",\"peak_vram_mib\":%" PRIu64 ",\"peak_ram_mib\":%" PRIu64
        ",\"median_peak_vram_mib\":%" PRIu64 ",\"median_peak_ram_mib\":%" PRIu64
        ",\"peak_memory_aggregation\":\"worst\",\"memory_measurement\":\"%s\",\"output_match\":%s,"
        "\"repetition_outputs_match\":%s,\"quality\":null,\"generated_output\":\"%s\",\"generated_token_ids\":[%s]}\n",
        json_escape(c.model_path).c_str(), json_escape(revision).c_str(), json_escape(c.backend).c_str(),
        json_escape(dev.name).c_str(), pt, gt, c.warmup, c.repetitions, fmt3(prefill * 1e3).c_str(),
        fmt3(decode * 1e3).c_str(), fmt3(rate(pt, prefill)).c_str(), fmt3(rate(gt, decode)).c_str(),
        fmt3(rate(pt + gt, prefill + decode)).c_str(), ws_mib, mapped, st.peak_active_weight_bytes, plan.state_bytes,
        plan.scratch_bytes, peak_v, peak_r, median(vram), median(ram), label.c_str(), option_bool(match),
        reps_match ? "true" : "false", json_escape(out).c_str(), ids.c_str());
  }
  return match == std::optional<bool>(false) ? 2 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  std::vector<std::string> args(argv + 1, argv + argc);
  std::optional<Config> cfg;
  try {
    cfg = parse_args(args);
  } catch (const ParseError& e) {
    std::fprintf(stderr, "error: %s\n\n%s\n", e.msg.c_str(), kUsage);
    return 1;
  }
  if (!cfg) {
    std::printf("%s\n", kUsage);
    return 0;
  }
  try {
    return cfg->backend == "mock" ? run_mock(*cfg) : run_cuda(*cfg);
  } catch (const Failure& f) {
    std::fprintf(stderr, "error: %s\n", f.msg.c_str());
    return 1;
  }
}
