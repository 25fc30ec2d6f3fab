// GGUF container index shared by the reader (gguf.cu) and the model loader.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

struct si_gguf;

namespace si {

constexpr uint64_t kGgufPreview = 3;  // array elements kept for the inspection summary

// One metadata value (GgufValue, model.rs:583-600). Arrays keep their element
// type, their length and their first kGgufPreview elements: decode reads no
// array contents.
struct GgufValue {
  uint32_t type = 0, elem_type = 0;
  uint64_t u = 0, count = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  std::vector<GgufValue> preview;
};

// summarize (src/bin/si-gguf-inspect.rs:84-101) of one value, with Rust's
// Debug formatting of the variants.
std::string gguf_summary(const GgufValue& v);

// One tensor-index entry with its resolved byte range (GgufTensorInfo).
struct GgufTensor {
  std::string name;
  uint32_t ndim = 0, type = 0;
  std::vector<uint64_t> dims;
  uint64_t offset = 0, data_start = 0, data_len = 0;
};

bool gguf_is_unsigned(const GgufValue& v);
int gguf_parse(const char* path, si_gguf** out, std::string* err);
int gguf_read(const si_gguf* g, uint64_t offset, void* dst, uint64_t bytes, std::string* err);
const GgufValue* gguf_meta(const si_gguf* g, const std::string& key);

}  // namespace si

struct si_gguf {
  std::string path;
  int fd = -1;
  uint32_t version = 0;
  uint64_t file_size = 0;
  std::map<std::string, si::GgufValue> meta;
  std::vector<si::GgufTensor> tensors;
  std::map<std::string, uint64_t> index;
  mutable std::map<std::string, std::string> summaries;  // si_gguf_meta_summary results
};
