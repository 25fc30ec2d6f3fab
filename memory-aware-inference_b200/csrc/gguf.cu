// GGUF container reader (host code): header, typed metadata and tensor index
// of a GGUF v2/v3 file, parsed as the reference does (src/model.rs:1033-1120
// parse_gguf, 1155-1205 GgufReader), and the qwen35 execution config derived
// from its metadata (src/model.rs:350-417 GgufQwen35Config::from_metadata).
// Tensor payloads are never held here: callers read row ranges with pread.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <memory>
#include <set>
#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iterator>
#include <map>
#include <string>
#include <vector>

#include "../../include/si_cuda.h"
#include "gguf.h"
#include "fault.h"

namespace si {
int fail(si_ctx* ctx, int code, const std::string& msg);
}

namespace {

// Strict UTF-8 check (String::from_utf8 in GgufReader::read_string).
bool valid_utf8(const std::string& s) {
  const unsigned char* p = reinterpret_cast<const unsigned char*>(s.data());
  size_t n = s.size(), i = 0;
  while (i < n) {
    unsigned c = p[i];
    if (c < 0x80) { ++i; continue; }
    int len = (c >= 0xC2 && c <= 0xDF) ? 2 : (c >= 0xE0 && c <= 0xEF) ? 3 : (c >= 0xF0 && c <= 0xF4) ? 4 : 0;
    if (!len || i + len > n) return false;
    unsigned c1 = p[i + 1];
    if (c == 0xE0 && c1 < 0xA0) return false;   // overlong
    if (c == 0xED && c1 > 0x9F) return false;   // surrogates
    if (c == 0xF0 && c1 < 0x90) return false;   // overlong
    if (c == 0xF4 && c1 > 0x8F) return false;   // above U+10FFFF
    for (int k = 1; k < len; ++k)
      if ((p[i + k] & 0xC0) != 0x80) return false;
    i += len;
  }
  return true;
}

// Sequential reader over the file with bounds checks (GgufReader).
struct Reader {
  FILE* f;
  uint64_t size, offset = 0;
  std::string err;
  bool read(void* dst, uint64_t n) {
    if (!err.empty()) return false;
    if (n > size || offset > size - n) {
      err = "GGUF header is truncated";
      return false;
    }
    if (n && (si::fault_fire(SI_FAULT_FILE_READ) || fread(dst, 1, n, f) != n)) {
      err = "GGUF read failed";
      return false;
    }
    offset += n;
    return true;
  }
  bool skip(uint64_t n) {
    if (!err.empty()) return false;
    if (n > size || offset > size - n) {
      err = "GGUF header is truncated";
      return false;
    }
    if (fseeko(f, off_t(n), SEEK_CUR) != 0) {
      err = "GGUF seek failed";
      return false;
    }
    offset += n;
    return true;
  }
  template <typename T>
  bool pod(T* v) {
    return read(v, sizeof(T));
  }
  bool str(std::string* s) {
    uint64_t n = 0;
    if (!pod(&n)) return false;
    if (n > size - offset) {
      err = "GGUF header is truncated";
      return false;
    }
    s->resize(n);
    if (!read(s->data(), n)) return false;
    if (!valid_utf8(*s)) {
      err = "GGUF string is not UTF-8";
      return false;
    }
    return true;
  }
};

// Element size of the fixed-size metadata value types, 0 for string/array.
uint64_t value_size(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
  }
}

bool read_value(Reader& r, uint32_t type, si::GgufValue* v, int depth) {
  v->type = type;
  switch (type) {
    case 0: { uint8_t x; if (!r.pod(&x)) return false; v->u = x; v->i = x; v->f = x; return true; }
    case 1: { int8_t x; if (!r.pod(&x)) return false; v->i = x; v->u = uint64_t(int64_t(x)); v->f = x; return true; }
    case 2: { uint16_t x; if (!r.pod(&x)) return false; v->u = x; v->i = x; v->f = x; return true; }
    case 3: { int16_t x; if (!r.pod(&x)) return false; v->i = x; v->u = uint64_t(int64_t(x)); v->f = x; return true; }
    case 4: { uint32_t x; if (!r.pod(&x)) return false; v->u = x; v->i = x; v->f = x; return true; }
    case 5: { int32_t x; if (!r.pod(&x)) return false; v->i = x; v->u = uint64_t(int64_t(x)); v->f = x; return true; }
    case 6: { float x; if (!r.pod(&x)) return false; v->f = x; return true; }
    case 7: { uint8_t x; if (!r.pod(&x)) return false; v->u = x != 0; v->i = x != 0; return true; }
    case 8: return r.str(&v->s);
    case 9: {
      uint32_t et = 0;
      uint64_t count = 0;
      if (!r.pod(&et) || !r.pod(&count)) return false;
      if (depth > 4) {
        r.err = "GGUF arrays nest too deeply";
        return false;
      }
      v->elem_type = et;
      v->count = count;
      const uint64_t es = value_size(et);
      if (count == 0) return true;  // element type is never read
      // the first elements are kept as a preview (the inspection summary);
      // decode needs only the length
      const uint64_t keep = std::min<uint64_t>(count, si::kGgufPreview);
      if (es) {  // fixed-size elements: the rest are skipped
        if (count > r.size / es) {
          r.err = "GGUF header is truncated";
          return false;
        }
        for (uint64_t i = 0; i < keep; ++i) {
          v->preview.emplace_back();
          if (!read_value(r, et, &v->preview.back(), depth + 1)) return false;
        }
        return r.skip((count - keep) * es);
      }
      if (et != 8 && et != 9) {
        r.err = "unsupported GGUF metadata type " + std::to_string(et);
        return false;
      }
      for (uint64_t i = 0; i < count; ++i) {
        si::GgufValue e;
        if (!read_value(r, et, &e, depth + 1)) return false;
        if (i < keep) v->preview.push_back(std::move(e));
      }
      return true;
    }
    case 10: { uint64_t x; if (!r.pod(&x)) return false; v->u = x; v->i = int64_t(x); v->f = double(x); return true; }
    case 11: { int64_t x; if (!r.pod(&x)) return false; v->i = x; v->u = uint64_t(x); v->f = double(x); return true; }
    case 12: { double x; if (!r.pod(&x)) return false; v->f = x; return true; }
    default:
      r.err = "unsupported GGUF metadata type " + std::to_string(type);
      return false;
  }
}

}  // namespace

namespace si {

// U8/U16/U32/U64: the types required_u32 (model.rs:454-469) accepts.
bool gguf_is_unsigned(const GgufValue& v) { return v.type == 0 || v.type == 2 || v.type == 4 || v.type == 10; }

int gguf_parse(const char* path, si_gguf** out, std::string* err) {
  *out = nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) {
    *err = std::string("open GGUF model ") + path + ": " + std::strerror(errno);
    return SI_E_INVALID;
  }
  struct stat st;
  if (fstat(fileno(f), &st) != 0) {
    *err = std::string("stat GGUF model ") + path + ": " + std::strerror(errno);
    fclose(f);
    return SI_E_INVALID;
  }
  Reader r{f, uint64_t(st.st_size), 0, {}};
  auto g = new si_gguf();
  g->path = path;
  g->file_size = uint64_t(st.st_size);
  auto bad = [&](const std::string& msg) {
    *err = msg;
    fclose(f);
    delete g;
    return SI_E_INVALID;
  };
  char magic[4];
  if (!r.read(magic, 4)) return bad(r.err);
  if (std::memcmp(magic, "GGUF", 4) != 0) return bad("GGUF header has invalid magic");
  uint32_t version = 0;
  uint64_t ntensors = 0, nmeta = 0;
  if (!r.pod(&version)) return bad(r.err);
  if (version != 2 && version != 3) return bad("unsupported GGUF version " + std::to_string(version));
  if (!r.pod(&ntensors) || !r.pod(&nmeta)) return bad(r.err);
  g->version = version;
  for (uint64_t i = 0; i < nmeta; ++i) {
    std::string key;
    uint32_t type = 0;
    GgufValue v;
    if (!r.str(&key) || !r.pod(&type) || !read_value(r, type, &v, 0)) return bad(r.err);
    if (!g->meta.emplace(key, v).second) return bad("GGUF metadata contains duplicate keys");
  }
  g->tensors.reserve(std::min<uint64_t>(ntensors, r.size / 24));  // an entry takes 24 B at least
  for (uint64_t i = 0; i < ntensors; ++i) {
    g->tensors.emplace_back();
    GgufTensor& t = g->tensors.back();
    uint32_t nd = 0;
    if (!r.str(&t.name) || !r.pod(&nd)) return bad(r.err);
    if (nd > (r.size - r.offset) / 8) return bad("GGUF header is truncated");
    t.ndim = nd;
    t.dims.resize(nd);
    for (uint32_t d = 0; d < nd; ++d)
      if (!r.pod(&t.dims[d])) return bad(r.err);
    if (!r.pod(&t.type) || !r.pod(&t.offset)) return bad(r.err);
    g->index[t.name] = i;  // a later entry of the same name wins (BTreeMap collect)
  }
  uint64_t alignment = 32;
  auto it = g->meta.find("general.alignment");
  if (it != g->meta.end() && (it->second.type == 4 || it->second.type == 10)) alignment = it->second.u;
  if (alignment == 0 || (alignment & (alignment - 1))) return bad("GGUF alignment must be a non-zero power of two");
  const uint64_t data_base = (r.offset + alignment - 1) / alignment * alignment;
  // a tensor's bytes run from its offset to the next tensor's (by offset) or
  // to the end of the file
  std::vector<uint64_t> order(ntensors);
  for (uint64_t i = 0; i < ntensors; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(),  // sort_by_key is stable
            [&](uint64_t a, uint64_t b) { return g->tensors[a].offset < g->tensors[b].offset; });
  for (uint64_t k = 0; k < ntensors; ++k) {
    GgufTensor& t = g->tensors[order[k]];
    if (t.offset > g->file_size || data_base > g->file_size - t.offset)
      return bad("GGUF tensor " + t.name + " exceeds file size");
    const uint64_t start = data_base + t.offset;
    const uint64_t end = k + 1 < ntensors ? data_base + g->tensors[order[k + 1]].offset : g->file_size;
    if (start > end || end > g->file_size) return bad("GGUF tensor " + t.name + " exceeds file size");
    t.data_start = start;
    t.data_len = end - start;
  }
  fclose(f);
  g->fd = open(path, O_RDONLY);
  if (g->fd < 0) return bad(std::string("open GGUF model ") + path + ": " + std::strerror(errno));
  *out = g;
  return SI_OK;
}

int gguf_read(const si_gguf* g, uint64_t offset, void* dst, uint64_t bytes, std::string* err) {
  uint8_t* p = static_cast<uint8_t*>(dst);
  while (bytes) {
    const ssize_t got = si::fault_fire(SI_FAULT_FILE_READ)
                            ? 0
                            : pread(g->fd, p, size_t(std::min<uint64_t>(bytes, uint64_t(1) << 30)), off_t(offset));
    if (got <= 0) {
      *err = "GGUF read of " + g->path + " failed: " + (got < 0 ? std::strerror(errno) : "unexpected end of file");
      return SI_E_INVALID;
    }
    p += got;
    offset += uint64_t(got);
    bytes -= uint64_t(got);
  }
  return SI_OK;
}

namespace {

// Rust's Debug of a float: the shortest digits that read back to the same
// value; exponential form ("1e-6", "1.5e20") when |x| < 1e-4 or |x| >= 1e16,
// else decimal with at least one fractional digit ("10000000.0", "0.1").
std::string rust_float_debug(double x, bool is_f32) {
  if (std::isnan(x)) return "NaN";
  if (std::isinf(x)) return x < 0 ? "-inf" : "inf";
  if (x == 0) return std::signbit(x) ? "-0.0" : "0.0";
  char buf[64];
  int p = 1;
  for (; p <= 17; ++p) {
    std::snprintf(buf, sizeof(buf), "%.*e", p - 1, x);
    const double back = std::strtod(buf, nullptr);
    if (is_f32 ? float(back) == float(x) : back == x) break;
  }
  // buf = [-]D[.DDD]e[+-]XX
  std::string t = buf, digits;
  const size_t epos = t.find('e');
  for (size_t i = 0; i < epos; ++i)
    if (std::isdigit(static_cast<unsigned char>(t[i]))) digits += t[i];
  const int e10 = std::atoi(t.c_str() + epos + 1);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  const double ax = std::fabs(x);
  const bool expo = is_f32 ? (float(ax) < 1e-4f || float(ax) >= 1e16f) : (ax < 1e-4 || ax >= 1e16);
  std::string out = x < 0 ? "-" : "";
  if (expo) {
    out += digits.substr(0, 1);
    if (digits.size() > 1) out += "." + digits.substr(1);
    out += "e" + std::to_string(e10);
  } else if (e10 >= 0) {
    std::string ip = digits.substr(0, std::min<size_t>(digits.size(), size_t(e10) + 1));
    while (ip.size() < size_t(e10) + 1) ip += '0';
    const std::string fp = digits.size() > size_t(e10) + 1 ? digits.substr(size_t(e10) + 1) : "0";
    out += ip + "." + fp;
  } else {
    out += "0." + std::string(size_t(-e10 - 1), '0') + digits;
  }
  return out;
}

// Rust's Debug of a str: quoted, with \t \r \n \0 \\ \" escaped and other
// control characters as \u{..}; other characters as they are.
std::string rust_str_debug(const std::string& v) {
  std::string o = "\"";
  for (unsigned char ch : v) {
    switch (ch) {
      case '\t': o += "\\t"; break;
      case '\r': o += "\\r"; break;
      case '\n': o += "\\n"; break;
      case '\0': o += "\\0"; break;
      case '\\': o += "\\\\"; break;
      case '"': o += "\\\""; break;
      default:
        if (ch < 0x20 || ch == 0x7f) {
          char b[16];
          std::snprintf(b, sizeof(b), "\\u{%x}", ch);
          o += b;
        } else {
          o += char(ch);
        }
    }
  }
  return o + "\"";
}

// The first `n` characters (Unicode scalar values) of UTF-8 text.
std::string utf8_prefix(const std::string& v, size_t n) {
  size_t i = 0, chars = 0;
  while (i < v.size() && chars < n) {
    const unsigned char c = static_cast<unsigned char>(v[i]);
    i += c < 0x80 ? 1 : c < 0xE0 ? 2 : c < 0xF0 ? 3 : 4;
    ++chars;
  }
  return v.substr(0, std::min(i, v.size()));
}

}  // namespace

std::string gguf_summary(const GgufValue& v) {
  switch (v.type) {
    case 0: return "U8(" + std::to_string(v.u) + ")";
    case 1: return "I8(" + std::to_string(v.i) + ")";
    case 2: return "U16(" + std::to_string(v.u) + ")";
    case 3: return "I16(" + std::to_string(v.i) + ")";
    case 4: return "U32(" + std::to_string(v.u) + ")";
    case 5: return "I32(" + std::to_string(v.i) + ")";
    case 6: return "F32(" + rust_float_debug(v.f, true) + ")";
    case 7: return std::string("Bool(") + (v.u ? "true" : "false") + ")";
    case 8: {
      if (v.s.size() > 160)
        return "string(len=" + std::to_string(v.s.size()) + ", prefix=" + rust_str_debug(utf8_prefix(v.s, 160)) + ")";
      return "string(" + rust_str_debug(v.s) + ")";
    }
    case 9: {
      std::string o = "array(len=" + std::to_string(v.count) + ", first=[";
      for (size_t k = 0; k < v.preview.size(); ++k) o += (k ? ", " : "") + gguf_summary(v.preview[k]);
      return o + "])";
    }
    case 10: return "U64(" + std::to_string(v.u) + ")";
    case 11: return "I64(" + std::to_string(v.i) + ")";
    case 12: return "F64(" + rust_float_debug(v.f, false) + ")";
    default: return "?";
  }
}

const GgufValue* gguf_meta(const si_gguf* g, const std::string& key) {
  auto it = g->meta.find(key);
  return it == g->meta.end() ? nullptr : &it->second;
}

}  // namespace si

// ---- C ABI -------------------------------------------------------------------
extern "C" {

int si_gguf_open(const char* path, si_gguf** out) {
  if (!path || !out) return si::fail(nullptr, SI_E_INVALID, "invalid GGUF arguments");
  std::string err;
  int rc = si::gguf_parse(path, out, &err);
  return rc ? si::fail(nullptr, rc, err) : SI_OK;
}

void si_gguf_close(si_gguf* g) {
  if (!g) return;
  if (g->fd >= 0) close(g->fd);
  delete g;
}

int si_gguf_info(const si_gguf* g, uint32_t* version, uint64_t* tensor_count, uint64_t* metadata_count) {
  if (!g) return SI_E_INVALID;
  if (version) *version = g->version;
  if (tensor_count) *tensor_count = g->tensors.size();
  if (metadata_count) *metadata_count = g->meta.size();
  return SI_OK;
}

int si_gguf_tensor_info(const si_gguf* g, uint64_t index, const char** name, uint32_t* ndim, uint64_t* dims,
                        uint32_t* ggml_type, uint64_t* data_start, uint64_t* data_len) {
  if (!g || index >= g->tensors.size()) return si::fail(nullptr, SI_E_INVALID, "GGUF tensor index out of range");
  const si::GgufTensor& t = g->tensors[index];
  if (name) *name = t.name.c_str();
  if (ndim) *ndim = t.ndim;
  if (dims)
    for (uint32_t d = 0; d < 4; ++d) dims[d] = d < t.ndim ? t.dims[d] : 1;  // first 4 of ndim
  if (ggml_type) *ggml_type = t.type;
  if (data_start) *data_start = t.data_start;
  if (data_len) *data_len = t.data_len;
  return SI_OK;
}

int si_gguf_find_tensor(const si_gguf* g, const char* name, uint64_t* index) {
  if (!g || !name || !index) return SI_E_INVALID;
  auto it = g->index.find(name);
  if (it == g->index.end()) return si::fail(nullptr, SI_E_INVALID, std::string("unknown GGUF tensor ") + name);
  *index = it->second;
  return SI_OK;
}

int si_gguf_meta_u64(const si_gguf* g, const char* key, uint64_t* out) {
  const si::GgufValue* v = g && key ? si::gguf_meta(g, key) : nullptr;
  if (!v) return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata is missing ") + (key ? key : ""));
  if (!si::gguf_is_unsigned(*v))
    return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata ") + key + " has unexpected value");
  *out = v->u;
  return SI_OK;
}

int si_gguf_meta_f64(const si_gguf* g, const char* key, double* out) {
  const si::GgufValue* v = g && key ? si::gguf_meta(g, key) : nullptr;
  if (!v) return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata is missing ") + (key ? key : ""));
  if (v->type != 6 && v->type != 12)
    return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata ") + key + " has unexpected value");
  *out = v->f;
  return SI_OK;
}

int si_gguf_meta_string(const si_gguf* g, const char* key, const char** out) {
  const si::GgufValue* v = g && key ? si::gguf_meta(g, key) : nullptr;
  if (!v) return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata is missing ") + (key ? key : ""));
  if (v->type != 8) return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata ") + key + " has unexpected value");
  *out = v->s.c_str();
  return SI_OK;
}

int si_gguf_meta_array_len(const si_gguf* g, const char* key, uint64_t* out) {
  const si::GgufValue* v = g && key ? si::gguf_meta(g, key) : nullptr;
  if (!v) return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata is missing ") + (key ? key : ""));
  if (v->type != 9) return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata ") + key + " has unexpected value");
  *out = v->count;
  return SI_OK;
}

int si_gguf_read(const si_gguf* g, uint64_t index, uint64_t offset, void* dst, uint64_t bytes) {
  if (!g || (!dst && bytes) || index >= g->tensors.size()) return si::fail(nullptr, SI_E_INVALID, "invalid GGUF read");
  const si::GgufTensor& t = g->tensors[index];
  if (offset > t.data_len || bytes > t.data_len - offset)
    return si::fail(nullptr, SI_E_INVALID, "GGUF read beyond tensor " + t.name);
  std::string err;
  int rc = si::gguf_read(g, t.data_start + offset, dst, bytes, &err);
  return rc ? si::fail(nullptr, rc, err) : SI_OK;
}

}  // extern "C"

// A layer's payloads packed for staging (StagedQwenLayer, model.rs:588-592).
struct si_gguf_packed {
  std::vector<uint8_t> bytes;
  std::vector<std::string> names;  // sorted, as the reference's BTreeMap
  std::vector<uint64_t> starts, ends;
};

extern "C" {

int si_gguf_stage_layer_packed(const si_gguf* g, uint32_t layer, const char* const* excluded, uint32_t n_excluded,
                               si_gguf_packed** out) {
  if (!g || !out || (n_excluded && !excluded)) return si::fail(nullptr, SI_E_INVALID, "invalid staging arguments");
  *out = nullptr;
  std::set<std::string> skip;
  for (uint32_t i = 0; i < n_excluded; ++i)
    if (excluded[i]) skip.insert(excluded[i]);
  const std::string prefix = "blk." + std::to_string(layer) + ".";
  // the layer's quantized tensors in name order, then stably by file offset
  std::vector<const si::GgufTensor*> infos;
  for (const auto& kv : g->index) {
    const si::GgufTensor& t = g->tensors[kv.second];
    if (kv.first.compare(0, prefix.size(), prefix) == 0 && !skip.count(kv.first) && t.type != 0) infos.push_back(&t);
  }
  std::stable_sort(infos.begin(), infos.end(),
                   [](const si::GgufTensor* a, const si::GgufTensor* b) { return a->data_start < b->data_start; });
  // nearby payloads are read together: a tensor starting within 4096 bytes
  // of the current run's end extends it
  std::vector<std::pair<uint64_t, uint64_t>> runs;
  for (const si::GgufTensor* t : infos) {
    const uint64_t end = t->data_start + t->data_len;
    if (!runs.empty() && t->data_start <= runs.back().second + 4096)
      runs.back().second = std::max(runs.back().second, end);
    else
      runs.push_back({t->data_start, end});
  }
  uint64_t total = 0;
  for (const auto& r : runs) total += r.second - r.first;  // runs lie inside the file
  auto p = std::make_unique<si_gguf_packed>();
  p->bytes.resize(total);
  std::map<std::string, std::pair<uint64_t, uint64_t>> ranges;
  uint64_t off = 0;
  for (const auto& r : runs) {
    std::string err;
    if (int rc = si::gguf_read(g, r.first, p->bytes.data() + off, r.second - r.first, &err))
      return si::fail(nullptr, rc, "read packed staged layer: " + err);
    for (const si::GgufTensor* t : infos)
      if (t->data_start >= r.first && t->data_start + t->data_len <= r.second) {
        const uint64_t a = off + (t->data_start - r.first);
        ranges[t->name] = {a, a + t->data_len};
      }
    off += r.second - r.first;
  }
  for (const auto& kv : ranges) {
    p->names.push_back(kv.first);
    p->starts.push_back(kv.second.first);
    p->ends.push_back(kv.second.second);
  }
  *out = p.release();
  return SI_OK;
}

int si_gguf_packed_info(const si_gguf_packed* p, const void** bytes, uint64_t* nbytes, uint32_t* n_ranges) {
  if (!p) return SI_E_INVALID;
  if (bytes) *bytes = p->bytes.data();
  if (nbytes) *nbytes = p->bytes.size();
  if (n_ranges) *n_ranges = uint32_t(p->names.size());
  return SI_OK;
}

int si_gguf_packed_range(const si_gguf_packed* p, uint32_t i, const char** name, uint64_t* start, uint64_t* end) {
  if (!p || i >= p->names.size()) return si::fail(nullptr, SI_E_INVALID, "staged range index out of range");
  if (name) *name = p->names[i].c_str();
  if (start) *start = p->starts[i];
  if (end) *end = p->ends[i];
  return SI_OK;
}

void si_gguf_packed_free(si_gguf_packed* p) { delete p; }

int si_gguf_advise_layer(const si_gguf* g, uint32_t layer, uint64_t* advised) {
  if (!g) return si::fail(nullptr, SI_E_INVALID, "invalid advise arguments");
  const long page = sysconf(_SC_PAGESIZE);
  if (page <= 0) return si::fail(nullptr, SI_E_INVALID, "page size is invalid");
  const uint64_t ps = uint64_t(page);
  const std::string prefix = "blk." + std::to_string(layer) + ".";
  uint64_t total = 0;
  for (const auto& kv : g->index) {
    if (kv.first.compare(0, prefix.size(), prefix) != 0) continue;
    const si::GgufTensor& t = g->tensors[kv.second];
    const uint64_t a = t.data_start & ~(ps - 1), b = (t.data_start + t.data_len + ps - 1) & ~(ps - 1);
    if (b <= a) continue;
    (void)posix_fadvise(g->fd, off_t(a), off_t(b - a), POSIX_FADV_WILLNEED);  // a hint: its result is not an error
    total += b - a;
  }
  if (advised) *advised = total;
  return SI_OK;
}

}  // extern "C"

namespace {

// A strict reader of one JSON document whose top level is an object: the
// string-valued top-level fields are returned, every other value is checked
// and skipped (the manifest test of detect_model_format, model.rs:46-62).
struct JsonReader {
  const std::string& s;
  size_t i = 0;
  std::string err;
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  bool fail_at(const char* what) {
    if (err.empty()) err = std::string("invalid model manifest JSON: ") + what + " at byte " + std::to_string(i);
    return false;
  }
  bool str(std::string* out) {
    if (i >= s.size() || s[i] != '"') return fail_at("expected a string");
    ++i;
    while (i < s.size() && s[i] != '"') {
      char ch = s[i++];
      if (static_cast<unsigned char>(ch) < 0x20) return fail_at("control character in a string");
      if (ch == '\\') {
        if (i >= s.size()) return fail_at("unterminated escape");
        const char e = s[i++];
        switch (e) {
          case '"': ch = '"'; break;
          case '\\': ch = '\\'; break;
          case '/': ch = '/'; break;
          case 'b': ch = '\b'; break;
          case 'f': ch = '\f'; break;
          case 'n': ch = '\n'; break;
          case 'r': ch = '\r'; break;
          case 't': ch = '\t'; break;
          case 'u': {
            if (i + 4 > s.size()) return fail_at("short unicode escape");
            for (int k = 0; k < 4; ++k)
              if (!std::isxdigit(static_cast<unsigned char>(s[i + k]))) return fail_at("bad unicode escape");
            const unsigned cp = unsigned(std::stoul(s.substr(i, 4), nullptr, 16));
            i += 4;
            if (out) {  // the fields compared here are ASCII; other code points are kept as UTF-8
              if (cp < 0x80) {
                out->push_back(char(cp));
              } else if (cp < 0x800) {
                out->push_back(char(0xC0 | (cp >> 6)));
                out->push_back(char(0x80 | (cp & 63)));
              } else {
                out->push_back(char(0xE0 | (cp >> 12)));
                out->push_back(char(0x80 | ((cp >> 6) & 63)));
                out->push_back(char(0x80 | (cp & 63)));
              }
            }
            continue;
          }
          default:
            return fail_at("bad escape");
        }
      }
      if (out) out->push_back(ch);
    }
    if (i >= s.size()) return fail_at("unterminated string");
    ++i;
    return true;
  }
  bool value(int depth, std::string* as_string, bool* is_string) {
    if (depth > 64) return fail_at("nesting too deep");
    ws();
    if (i >= s.size()) return fail_at("expected a value");
    const char ch = s[i];
    if (is_string) *is_string = ch == '"';
    if (ch == '"') return str(as_string);
    if (ch == '{' || ch == '[') {
      const char close = ch == '{' ? '}' : ']';
      ++i;
      ws();
      if (i < s.size() && s[i] == close) {
        ++i;
        return true;
      }
      for (;;) {
        ws();
        if (ch == '{') {
          if (!str(nullptr)) return false;
          ws();
          if (i >= s.size() || s[i] != ':') return fail_at("expected ':'");
          ++i;
        }
        if (!value(depth + 1, nullptr, nullptr)) return false;
        ws();
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        if (i < s.size() && s[i] == close) {
          ++i;
          return true;
        }
        return fail_at("expected ',' or a closing bracket");
      }
    }
    for (const char* lit : {"true", "false", "null"})
      if (s.compare(i, std::strlen(lit), lit) == 0) {
        i += std::strlen(lit);
        return true;
      }
    // number: -?(0|[1-9][0-9]*)(.[0-9]+)?([eE][+-]?[0-9]+)?
    size_t j = i;
    if (j < s.size() && s[j] == '-') ++j;
    if (j >= s.size() || !std::isdigit(static_cast<unsigned char>(s[j]))) return fail_at("expected a value");
    if (s[j] == '0') ++j;
    else while (j < s.size() && std::isdigit(static_cast<unsigned char>(s[j]))) ++j;
    if (j < s.size() && s[j] == '.') {
      ++j;
      if (j >= s.size() || !std::isdigit(static_cast<unsigned char>(s[j]))) return fail_at("bad number");
      while (j < s.size() && std::isdigit(static_cast<unsigned char>(s[j]))) ++j;
    }
    if (j < s.size() && (s[j] == 'e' || s[j] == 'E')) {
      ++j;
      if (j < s.size() && (s[j] == '+' || s[j] == '-')) ++j;
      if (j >= s.size() || !std::isdigit(static_cast<unsigned char>(s[j]))) return fail_at("bad number");
      while (j < s.size() && std::isdigit(static_cast<unsigned char>(s[j]))) ++j;
    }
    i = j;
    return true;
  }
};

bool json_top_level_strings(const std::string& text, std::map<std::string, std::string>* out, std::string* err) {
  JsonReader r{text, 0, {}};
  r.ws();
  if (r.i >= text.size() || text[r.i] != '{') {
    *err = "invalid model manifest JSON: expected an object";
    return false;
  }
  ++r.i;
  r.ws();
  if (r.i < text.size() && text[r.i] == '}') {
    ++r.i;
  } else {
    for (;;) {
      std::string key;
      r.ws();
      if (!r.str(&key)) break;
      r.ws();
      if (r.i >= text.size() || text[r.i] != ':') {
        r.fail_at("expected ':'");
        break;
      }
      ++r.i;
      std::string v;
      bool is_str = false;
      if (!r.value(1, &v, &is_str)) break;
      if (is_str) (*out)[key] = v;
      r.ws();
      if (r.i < text.size() && text[r.i] == ',') {
        ++r.i;
        continue;
      }
      if (r.i < text.size() && text[r.i] == '}') {
        ++r.i;
        break;
      }
      r.fail_at("expected ',' or '}'");
      break;
    }
  }
  if (r.err.empty()) {
    r.ws();
    if (r.i != text.size()) r.fail_at("trailing characters");
  }
  if (!r.err.empty()) {
    *err = r.err;
    return false;
  }
  return true;
}

// GgufQwen35Config (model.rs:321-348) as read by from_metadata.
struct Qwen35Meta {
  uint64_t H, I, L, qh, kvh, kl, vl, ctxlen, interval, inner, state, groups, conv, rank, eos, vocab;
  float eps, theta;
};

// GgufQwen35Config::from_metadata (model.rs:350-417): the same keys, types,
// evaluation order and checks.
int qwen35_from_metadata(const si_gguf* g, Qwen35Meta* q) {
  const char* arch = nullptr;
  if (int rc = si_gguf_meta_string(g, "general.architecture", &arch)) return rc;
  if (std::string(arch) != "qwen35")
    return si::fail(nullptr, SI_E_UNSUPPORTED, std::string("unsupported GGUF architecture ") + arch + "; expected qwen35");
  double eps = 0, theta = 0;
  const struct {
    const char* key;
    uint64_t* dst;
  } ints[] = {{"qwen35.embedding_length", &q->H},         {"qwen35.feed_forward_length", &q->I},
              {"qwen35.block_count", &q->L},              {"qwen35.attention.head_count", &q->qh},
              {"qwen35.attention.head_count_kv", &q->kvh}, {"qwen35.attention.key_length", &q->kl},
              {"qwen35.attention.value_length", &q->vl},  {"qwen35.context_length", &q->ctxlen},
              {"tokenizer.ggml.eos_token_id", &q->eos},   {"qwen35.full_attention_interval", &q->interval},
              {"qwen35.ssm.inner_size", &q->inner},       {"qwen35.ssm.state_size", &q->state},
              {"qwen35.ssm.group_count", &q->groups},     {"qwen35.ssm.conv_kernel", &q->conv},
              {"qwen35.ssm.time_step_rank", &q->rank}};
  // required_u32 (model.rs:454-469): unsigned types only, and it must fit u32
  auto req_u32 = [&](const char* key, uint64_t* dst) -> int {
    if (int rc = si_gguf_meta_u64(g, key, dst)) return rc;
    if (*dst > 0xFFFFFFFFull) return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata ") + key + " overflows u32");
    return SI_OK;
  };
  for (const auto& e : ints) {
    if (e.dst == &q->ctxlen) {  // vocab and the floats come between these in from_metadata
      if (int rc = si_gguf_meta_array_len(g, "tokenizer.ggml.tokens", &q->vocab)) return rc;
    }
    if (e.dst == &q->eos) {
      if (int rc = si_gguf_meta_f64(g, "qwen35.attention.layer_norm_rms_epsilon", &eps)) return rc;
      if (int rc = si_gguf_meta_f64(g, "qwen35.rope.freq_base", &theta)) return rc;
    }
    if (int rc = req_u32(e.key, e.dst)) return rc;
  }
  q->eps = float(eps);
  q->theta = float(theta);
  if (!q->H || !q->I || !q->L || !q->qh || !q->kvh || !q->kl || !q->vl || !q->vocab || !q->ctxlen || !q->interval ||
      !q->inner || !q->state || !q->groups || !q->conv || !q->rank || !std::isfinite(q->eps) || q->eps <= 0.f ||
      !std::isfinite(q->theta) || q->theta <= 1.f)
    return si::fail(nullptr, SI_E_INVALID, "Qwen3.6 GGUF config contains invalid dimensions");
  if (q->qh % q->kvh)
    return si::fail(nullptr, SI_E_INVALID, "Qwen3.6 attention heads must be divisible by key/value heads");
  if (q->inner % q->state)
    return si::fail(nullptr, SI_E_INVALID, "Qwen3.6 SSM inner size must be divisible by state size");
  return SI_OK;
}

}  // namespace

extern "C" {

int si_gguf_qwen35_config(const si_gguf* g, uint32_t kv_capacity, si_model_config* c) {
  if (!g || !c) return si::fail(nullptr, SI_E_INVALID, "invalid GGUF config arguments");
  Qwen35Meta q;
  if (int rc = qwen35_from_metadata(g, &q)) return rc;
  uint64_t H = q.H, I = q.I, L = q.L, qh = q.qh, kvh = q.kvh, kl = q.kl, vl = q.vl, ctxlen = q.ctxlen,
           interval = q.interval, inner = q.inner, state = q.state, groups = q.groups, conv = q.conv, rank = q.rank,
           eos = q.eos, vocab = q.vocab, rot = 0;
  const float eps_f = q.eps, theta_f = q.theta;
  // the runtime reads the rotary width separately (qwen35_runtime.rs:811-813)
  {
    const si::GgufValue* v = si::gguf_meta(g, "qwen35.rope.dimension_count");
    if (!v || (v->type != 4 && v->type != 10) || v->u > 0xFFFFFFFFull)
      return si::fail(nullptr, SI_E_INVALID, "GGUF model is missing qwen35.rope.dimension_count");
    rot = v->u;
  }
  if (vocab > 0xFFFFFFFFull) return si::fail(nullptr, SI_E_INVALID, "Qwen3.6 GGUF vocabulary overflows u32");
  // one head width per attention layer and one dt/alpha/beta row per value head
  if (vl != kl) return si::fail(nullptr, SI_E_UNSUPPORTED, "attention value_length must equal key_length");
  if (rank != inner / state) return si::fail(nullptr, SI_E_UNSUPPORTED, "SSM time_step_rank must equal inner_size / state_size");
  si_model_config_qwen36_27b(c);
  c->hidden = uint32_t(H);
  c->intermediate = uint32_t(I);
  c->layers = uint32_t(L);
  c->vocab = uint32_t(vocab);
  c->attn_interval = uint32_t(interval);
  c->attn_q_heads = uint32_t(qh);
  c->attn_kv_heads = uint32_t(kvh);
  c->attn_head_dim = uint32_t(kl);
  c->rotary_dim = uint32_t(rot);
  c->rope_theta = theta_f;
  c->gdn_key_heads = uint32_t(groups);                  // ssm_key_heads (model.rs:419-421)
  c->gdn_value_heads = uint32_t(inner / state);         // ssm_value_heads (model.rs:424-426)
  c->gdn_head_dim = uint32_t(state);                    // ssm_key_dim / ssm_value_dim
  c->conv_kernel = uint32_t(conv);
  c->rms_eps = eps_f;
  c->eos_token = uint32_t(eos);
  c->kv_capacity = kv_capacity ? kv_capacity : uint32_t(std::min<uint64_t>(ctxlen, 4096));
  c->weight_init = 0;
  // the config's per-role types are those of the first layer / the head
  auto type_of = [&](const std::string& name, uint32_t* t) {
    auto it = g->index.find(name);
    if (it != g->index.end()) *t = g->tensors[it->second].type;
  };
  type_of("blk.0.ffn_gate.weight", &c->mlp_type);
  type_of("blk.0.ffn_down.weight", &c->down_type);
  type_of("output.weight", &c->head_type);
  return SI_OK;
}


int si_gguf_qwen35_layer_kind(const si_gguf* g, uint32_t layer, uint32_t* kind) {
  if (!g || !kind) return si::fail(nullptr, SI_E_INVALID, "invalid layer kind arguments");
  Qwen35Meta q;
  if (int rc = qwen35_from_metadata(g, &q)) return rc;
  if (layer >= q.L)
    return si::fail(nullptr, SI_E_INVALID, "Qwen3.6 layer " + std::to_string(layer) + " exceeds " +
                                               std::to_string(q.L) + " layers");
  const std::string pre = "blk." + std::to_string(layer);
  const bool has_delta = g->index.count(pre + ".ssm_a") != 0;
  const bool has_attn = g->index.count(pre + ".attn_q.weight") != 0;
  if (has_delta == has_attn)
    return si::fail(nullptr, SI_E_INVALID,
                    "Qwen3.6 layer " + std::to_string(layer) + " does not have exactly one execution kind");
  const bool want_attn = (uint64_t(layer) + 1) % q.interval == 0;
  if (has_attn != want_attn)
    return si::fail(nullptr, SI_E_INVALID, "Qwen3.6 layer " + std::to_string(layer) + " tensor kind " +
                                               (has_delta ? "GatedDeltaNet" : "FullAttention") +
                                               " disagrees with interval " + std::to_string(q.interval));
  *kind = has_attn ? SI_LAYER_FULL_ATTENTION : SI_LAYER_GATED_DELTA_NET;
  return SI_OK;
}

int si_gguf_tensor_payload(const si_gguf* g, uint64_t index, uint64_t* elements, uint64_t* expected_bytes,
                           uint32_t* known) {
  if (!g || index >= g->tensors.size()) return si::fail(nullptr, SI_E_INVALID, "GGUF tensor index out of range");
  const si::GgufTensor& t = g->tensors[index];
  // element_count (model.rs:512-518)
  uint64_t n = 1;
  for (uint64_t d : t.dims) {
    if (d && n > UINT64_MAX / d)
      return si::fail(nullptr, SI_E_INVALID, "GGUF tensor " + t.name + " element count overflows");
    n *= d;
  }
  if (elements) *elements = n;
  // expected_payload_bytes (model.rs:532-573): F32, F16/BF16 and the K-quants
  uint64_t bytes = 0;
  bool k = true;
  if (t.type == 0) {
    if (n > UINT64_MAX / 4) k = false;
    bytes = n * 4;
  } else if (t.type == 1 || t.type == 30) {
    if (n > UINT64_MAX / 2) k = false;
    bytes = n * 2;
  } else if (t.type == SI_GGML_TYPE_Q4_K || t.type == SI_GGML_TYPE_Q5_K || t.type == SI_GGML_TYPE_Q6_K) {
    const char* label = t.type == SI_GGML_TYPE_Q4_K ? "Q4_K" : t.type == SI_GGML_TYPE_Q5_K ? "Q5_K" : "Q6_K";
    if (n % 256)
      return si::fail(nullptr, SI_E_INVALID, std::string("GGUF ") + label + " tensor " + t.name + " has " +
                                                 std::to_string(n) + " elements; expected a multiple of 256");
    const uint64_t bb = t.type == SI_GGML_TYPE_Q4_K ? 144 : t.type == SI_GGML_TYPE_Q5_K ? 176 : 210;
    if (n / 256 > UINT64_MAX / bb) k = false;
    bytes = n / 256 * bb;
  } else {
    k = false;
  }
  if (expected_bytes) *expected_bytes = k ? bytes : 0;
  if (known) *known = k ? 1 : 0;
  return SI_OK;
}

int si_detect_model_format(const char* path, uint32_t* format) {
  if (!path || !format) return si::fail(nullptr, SI_E_INVALID, "invalid model format arguments");
  struct stat st;
  if (stat(path, &st) != 0) return si::fail(nullptr, SI_E_INVALID, std::string("stat model ") + path + ": " + std::strerror(errno));
  if (S_ISDIR(st.st_mode)) {
    // a BF16 Safetensors artifact: manifest.json with format "safetensors" and
    // dtype "bfloat16" (model.rs:46-62)
    const std::string manifest = std::string(path) + "/manifest.json";
    FILE* f = std::fopen(manifest.c_str(), "rb");
    if (!f) return si::fail(nullptr, SI_E_INVALID, "read model manifest " + manifest + ": " + std::strerror(errno));
    std::string text;
    char buf[4096];
    size_t got;
    while ((got = std::fread(buf, 1, sizeof(buf), f)) > 0) text.append(buf, got);
    std::fclose(f);
    std::map<std::string, std::string> fields;
    std::string err;
    if (!json_top_level_strings(text, &fields, &err)) return si::fail(nullptr, SI_E_INVALID, err);
    if (fields.count("format") && fields["format"] == "safetensors" && fields.count("dtype") &&
        fields["dtype"] == "bfloat16") {
      *format = SI_FORMAT_SAFETENSORS;
      return SI_OK;
    }
    return si::fail(nullptr, SI_E_INVALID, "model directory is not a BF16 Safetensors artifact");
  }
  FILE* f = std::fopen(path, "rb");
  if (!f) return si::fail(nullptr, SI_E_INVALID, std::string("open model ") + path + ": " + std::strerror(errno));
  char magic[4];
  const size_t n = std::fread(magic, 1, 4, f);
  std::fclose(f);
  if (n < 4) return si::fail(nullptr, SI_E_INVALID, "failed to fill whole buffer");  // read_exact's error
  if (std::memcmp(magic, "GGUF", 4) == 0) {
    *format = SI_FORMAT_GGUF;
    return SI_OK;
  }
  return si::fail(nullptr, SI_E_INVALID, std::string("unsupported model container ") + path +
                                             "; expected a Safetensors directory or GGUF file");
}


int si_gguf_meta_key_at(const si_gguf* g, uint64_t index, const char** key) {
  if (!g || !key || index >= g->meta.size()) return si::fail(nullptr, SI_E_INVALID, "GGUF metadata index out of range");
  auto it = g->meta.begin();
  std::advance(it, long(index));
  *key = it->first.c_str();
  return SI_OK;
}

int si_gguf_meta_summary(const si_gguf* g, const char* key, const char** out) {
  const si::GgufValue* v = g && key ? si::gguf_meta(g, key) : nullptr;
  if (!v || !out) return si::fail(nullptr, SI_E_INVALID, std::string("GGUF metadata is missing ") + (key ? key : ""));
  auto& slot = g->summaries[key];
  if (slot.empty()) slot = si::gguf_summary(*v);
  *out = slot.c_str();
  return SI_OK;
}

}  // extern "C"
