// si-gguf-inspect: the reference's GGUF inspection probe
// (src/bin/si-gguf-inspect.rs) over the C ABI: tensor count, the first Q4_K
// tensors, per-type counts, the special tensors, the first other tensors and
// every metadata key with its summarised value. Usage errors exit 2, open
// errors exit 1 (as the reference's probe).
#include <cinttypes>
#include <cstdio>
#include <map>
#include <optional>
#include <string>
#include <vector>

#include "si_cuda.h"

namespace {

struct Tensor {
  std::string name;
  uint32_t type = 0, ndim = 0;
  uint64_t dims[4] = {1, 1, 1, 1};
  uint64_t bytes = 0, elements = 0;
  uint64_t index = 0;
};

std::string shape(const Tensor& t) {  // Debug of Vec<usize>
  std::string s = "[";
  for (uint32_t d = 0; d < t.ndim && d < 4; ++d) s += (d ? ", " : "") + std::to_string(t.dims[d]);
  return s + "]";
}

// parse_model (si-gguf-inspect.rs:71-82): only "--model PATH" pairs
std::optional<std::string> parse_model(int argc, char** argv) {
  std::optional<std::string> model;
  for (int i = 1; i < argc; i += 2) {
    if (std::string(argv[i]) != "--model") return std::nullopt;
    model = i + 1 < argc ? std::optional<std::string>(argv[i + 1]) : std::nullopt;
  }
  return model;
}

}  // namespace

int main(int argc, char** argv) {
  const std::optional<std::string> model = parse_model(argc, argv);
  if (!model) {
    std::fprintf(stderr, "Usage: si-gguf-inspect --model PATH\n");
    return 2;
  }
  si_gguf* g = nullptr;
  if (si_gguf_open(model->c_str(), &g) != SI_OK) {
    std::fprintf(stderr, "error: %s\n", si_global_last_error());
    return 1;
  }
  uint32_t version = 0;
  uint64_t ntensors = 0, nmeta = 0;
  si_gguf_info(g, &version, &ntensors, &nmeta);
  // the store's tensors by name; a later entry of a repeated name wins
  std::map<std::string, Tensor> byname;
  for (uint64_t i = 0; i < ntensors; ++i) {
    Tensor t;
    const char* name = nullptr;
    uint64_t start = 0;
    si_gguf_tensor_info(g, i, &name, &t.ndim, t.dims, &t.type, &start, &t.bytes);
    t.name = name ? name : "";
    t.index = i;
    uint32_t known = 0;
    if (si_gguf_tensor_payload(g, i, &t.elements, nullptr, &known) != SI_OK) t.elements = 0;
    byname[t.name] = t;
  }
  std::printf("model=%s\n", model->c_str());
  std::printf("tensors=%zu\n", byname.size());
  int shown = 0;
  for (const auto& kv : byname) {
    const Tensor& t = kv.second;
    if (t.type != SI_GGML_TYPE_Q4_K || shown >= 12) continue;
    ++shown;
    std::printf("q4_k_tensor=%s shape=%s bytes=%" PRIu64 " elements=%" PRIu64 "\n", t.name.c_str(), shape(t).c_str(),
                t.bytes, t.elements);
  }
  std::map<uint32_t, uint64_t> counts;
  for (const auto& kv : byname) counts[kv.second.type]++;
  std::string c = "{";
  for (const auto& kv : counts) c += (c.size() > 1 ? ", " : "") + std::to_string(kv.first) + ": " + std::to_string(kv.second);
  std::printf("tensor_type_counts=%s}\n", c.c_str());
  for (const char* name : {"token_embd.weight", "output.weight", "output_norm.weight"}) {
    auto it = byname.find(name);
    if (it == byname.end()) continue;
    std::printf("special_tensor=%s type=%u shape=%s bytes=%" PRIu64 "\n", name, it->second.type,
                shape(it->second).c_str(), it->second.bytes);
  }
  shown = 0;
  for (const auto& kv : byname) {
    const Tensor& t = kv.second;
    if (t.type == SI_GGML_TYPE_Q4_K || shown >= 24) continue;
    ++shown;
    std::printf("non_q4_tensor=%s type=%u shape=%s bytes=%" PRIu64 "\n", t.name.c_str(), t.type, shape(t).c_str(),
                t.bytes);
  }
  for (uint64_t i = 0; i < nmeta; ++i) {
    const char *key = nullptr, *summary = nullptr;
    if (si_gguf_meta_key_at(g, i, &key) != SI_OK || si_gguf_meta_summary(g, key, &summary) != SI_OK) continue;
    std::printf("metadata.%s=%s\n", key, summary);
  }
  si_gguf_close(g);
  return 0;
}
