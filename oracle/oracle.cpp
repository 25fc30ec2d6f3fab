// CPU oracle for the batch-1 K-quant decode hot path.
//
// TEST INFRASTRUCTURE ONLY. This file restates, in plain C++, the CPU code of
// vrlda/memory-aware-inference for the path that the CUDA backend replaces.
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
// reference arm may load it, and only as the checker or the timed CPU
// baseline. The product library never links or calls it.
//
// Parity pinning: the reference is Rust (no toolchain in this image) and its
// runtime is macOS/Metal-only, so it cannot be built or run here. This
// restatement is pinned against every known-answer test the reference holds
// for the path (src/quant.rs:213-280, src/qwen35.rs:232-296,
// src/cache.rs:173-291, src/metal.rs:7362-7602 and 8252-8404); those KATs are
// replayed in tests/test_oracle_kats.py. The KV-cache container the cache.rs
// tests exercise is restated in oracle/kv_cache.py.
//
// Floating point follows Rust semantics: IEEE binary32, no FMA contraction
// (build with -ffp-contract=off), left-to-right evaluation, sequential sums.
// Transcendentals come from glibc (expf, log1pf, sqrtf, powf, sinf, cosf),
// which is what Rust's f32 methods call on Linux.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <cstdlib>
#include <vector>
#include <algorithm>
#include <omp.h>

#include "../include/si_cuda.h"

namespace {

constexpr int kQK = 256;

// quant.rs:187-207 — f16 bits to f32, including subnormals.
float f16_to_f32(uint16_t bits) {
  uint32_t sign = uint32_t(bits & 0x8000u) << 16;
  uint32_t exponent = (bits >> 10) & 0x1f;
  uint32_t fraction = bits & 0x03ffu;
  uint32_t value;
  if (exponent == 0 && fraction == 0) {
    value = sign;
  } else if (exponent == 0) {
    int32_t e = -14;
    while ((fraction & 0x0400u) == 0) {
      fraction <<= 1;
      e -= 1;
    }
    fraction &= 0x03ffu;
    value = sign | (uint32_t(e + 127) << 23) | (fraction << 13);
  } else if (exponent == 0x1f) {
    value = sign | 0x7f800000u | (fraction << 13);
  } else {
    value = sign | ((exponent + 112) << 23) | (fraction << 13);
  }
  float out;
  std::memcpy(&out, &value, 4);
  return out;
}

uint16_t rd16(const uint8_t* p) { return uint16_t(p[0] | (p[1] << 8)); }

// quant.rs:176-185
void get_scale_min(int index, const uint8_t* scales, uint8_t* sc, uint8_t* mn) {
  if (index < 4) {
    *sc = scales[index] & 0x3f;
    *mn = scales[index + 4] & 0x3f;
  } else {
    *sc = (scales[index + 4] & 0x0f) | ((scales[index - 4] >> 6) << 4);
    *mn = (scales[index + 4] >> 4) | ((scales[index] >> 6) << 4);
  }
}

// quant.rs:36-63 — one Q4_K super-block (144 B) to 256 f32.
void deq_q4k_block(const uint8_t* block, float* out) {
  float d = f16_to_f32(rd16(block));
  float mn = f16_to_f32(rd16(block + 2));
  const uint8_t* scales = block + 4;
  const uint8_t* quants = block + 16;
  int si = 0;
  for (int g = 0; g < 4; ++g) {
    uint8_t s, m;
    get_scale_min(si, scales, &s, &m);
    float d1 = d * float(s);
    float m1 = mn * float(m);
    get_scale_min(si + 1, scales, &s, &m);
    float d2 = d * float(s);
    float m2 = mn * float(m);
    const uint8_t* q = quants + g * 32;
    for (int i = 0; i < 32; ++i) *out++ = d1 * float(q[i] & 0x0f) - m1;
    for (int i = 0; i < 32; ++i) *out++ = d2 * float(q[i] >> 4) - m2;
    si += 2;
  }
}

// quant.rs:87-123 — one Q5_K super-block (176 B).
void deq_q5k_block(const uint8_t* block, float* out) {
  float d = f16_to_f32(rd16(block));
  float mn = f16_to_f32(rd16(block + 2));
  const uint8_t* scales = block + 4;
  const uint8_t* high = block + 16;
  const uint8_t* quants = block + 48;
  uint8_t lo_mask = 1, hi_mask = 2;
  int si = 0;
  for (int g = 0; g < 4; ++g) {
    uint8_t s1, m1b, s2, m2b;
    get_scale_min(si, scales, &s1, &m1b);
    get_scale_min(si + 1, scales, &s2, &m2b);
    float d1 = d * float(s1);
    float m1 = mn * float(m1b);
    float d2 = d * float(s2);
    float m2 = mn * float(m2b);
    const uint8_t* q = quants + g * 32;
    for (int i = 0; i < 32; ++i) {
      int h = (high[i] & lo_mask) ? 16 : 0;
      *out++ = d1 * float((q[i] & 0x0f) + h) - m1;
    }
    for (int i = 0; i < 32; ++i) {
      int h = (high[i] & hi_mask) ? 16 : 0;
      *out++ = d2 * float((q[i] >> 4) + h) - m2;
    }
    si += 2;
    lo_mask <<= 2;
    hi_mask <<= 2;
  }
}

// quant.rs:145-172 — one Q6_K super-block (210 B).
void deq_q6k_block(const uint8_t* block, float* out) {
  const uint8_t* ql = block;
  const uint8_t* qh = block + 128;
  const int8_t* sc = reinterpret_cast<const int8_t*>(block + 192);
  float d = f16_to_f32(rd16(block + 208));
  for (int half = 0; half < 2; ++half) {
    const uint8_t* low = ql + half * 64;
    const uint8_t* high = qh + half * 32;
    const int8_t* bs = sc + half * 8;
    float* base = out + half * 128;
    for (int i = 0; i < 32; ++i) {
      int s = i / 16;
      uint8_t hb = high[i];
      int q1 = int((low[i] & 0x0f) | ((hb & 0x03) << 4)) - 32;
      int q2 = int((low[i + 32] & 0x0f) | (((hb >> 2) & 0x03) << 4)) - 32;
      int q3 = int((low[i] >> 4) | (((hb >> 4) & 0x03) << 4)) - 32;
      int q4 = int((low[i + 32] >> 4) | ((hb >> 6) << 4)) - 32;
      base[i] = d * float(bs[s]) * float(q1);
      base[i + 32] = d * float(bs[s + 2]) * float(q2);
      base[i + 64] = d * float(bs[s + 4]) * float(q3);
      base[i + 96] = d * float(bs[s + 6]) * float(q4);
    }
  }
}

int block_bytes(uint32_t type) {
  switch (type) {
    case SI_GGML_TYPE_Q4_K: return 144;
    case SI_GGML_TYPE_Q5_K: return 176;
    case SI_GGML_TYPE_Q6_K: return 210;
    case SI_GGML_TYPE_F32: return 4 * kQK;
    default: return 0;
  }
}

void deq_block(uint32_t type, const uint8_t* b, float* out) {
  switch (type) {
    case SI_GGML_TYPE_Q4_K: deq_q4k_block(b, out); break;
    case SI_GGML_TYPE_Q5_K: deq_q5k_block(b, out); break;
    case SI_GGML_TYPE_Q6_K: deq_q6k_block(b, out); break;
    case SI_GGML_TYPE_F32: std::memcpy(out, b, 4 * kQK); break;
  }
}

void deq_row(uint32_t type, const uint8_t* row, size_t cols, float* out) {
  int bb = block_bytes(type);
  for (size_t b = 0; b < cols / kQK; ++b) deq_block(type, row + b * bb, out + b * kQK);
}

size_t row_bytes(uint32_t type, size_t cols) {
  if (type == SI_GGML_TYPE_F32) return cols * 4;
  return cols / kQK * block_bytes(type);
}

// metal.rs:7476-7484 (the matvec test's CPU reference): dequantize, then a
// sequential f32 sum of w*x per row. Rows run in parallel; each row's order
// is the reference's. Eight rows are summed side by side, one super-block of
// columns at a time: each row keeps its own sequential chain (the same
// additions in the same order), the eight independent chains only let the
// core overlap them.
void matvec(uint32_t type, const uint8_t* w, size_t rows, size_t cols, const float* x,
            float* y, int threads) {
  constexpr size_t RG = 8;
  const size_t rb = row_bytes(type, cols), bb = size_t(block_bytes(type)), nb = cols / kQK;
  const long groups = long((rows + RG - 1) / RG);
#pragma omp parallel num_threads(threads)
  {
    std::vector<float> tmp(RG * kQK);
#pragma omp for schedule(static)
    for (long gi = 0; gi < groups; ++gi) {
      const size_t r0 = size_t(gi) * RG, nr = std::min(RG, rows - r0);
      float s[RG] = {};
      // F32 rows may end in a partial super-block of columns
      const size_t nbt = type == SI_GGML_TYPE_F32 ? (cols + kQK - 1) / kQK : nb;
      for (size_t b = 0; b < nbt; ++b) {
        const int len = int(std::min<size_t>(kQK, cols - b * kQK));
        const float* wr[RG];
        for (size_t r = 0; r < RG; ++r) {
          if (type == SI_GGML_TYPE_F32) {
            wr[r] = reinterpret_cast<const float*>(w + (r0 + std::min(r, nr - 1)) * rb) + b * kQK;
            continue;
          }
          deq_block(type, w + (r0 + std::min(r, nr - 1)) * rb + b * bb, tmp.data() + r * kQK);
          wr[r] = tmp.data() + r * kQK;
        }
        const float* xb = x + b * kQK;
        for (int c = 0; c < len; ++c) {
          const float xv = xb[c];
#pragma GCC unroll 8
          for (size_t r = 0; r < RG; ++r) s[r] += wr[r][c] * xv;
        }
      }
      for (size_t r = 0; r < nr; ++r) y[r0 + r] = s[r];
    }
  }
}

// qwen35.rs:8-10
float silu(float v) { return v / (1.0f + std::exp(-v)); }

// qwen35_runtime.rs:331-337
float softplus(float v) { return v > 20.0f ? v : std::log1p(std::exp(v)); }

// qwen35.rs:53-86 — (1+w) head RMSNorm.
void rms_norm_heads(const float* in, const float* w, size_t heads, size_t hd, float eps,
                    float* out) {
  for (size_t h = 0; h < heads; ++h) {
    const float* x = in + h * hd;
    float s = 0.0f;
    for (size_t i = 0; i < hd; ++i) s += x[i] * x[i];
    float inv = 1.0f / std::sqrt(s / float(hd) + eps);
    for (size_t i = 0; i < hd; ++i) out[h * hd + i] = x[i] * inv * (1.0f + w[i]);
  }
}

// qwen35.rs:14-49 — gated RMSNorm (weight w, not 1+w).
void gated_rms_norm(const float* in, const float* gate, const float* w, size_t heads,
                    size_t hd, float eps, float* out) {
  for (size_t h = 0; h < heads; ++h) {
    const float* x = in + h * hd;
    float s = 0.0f;
    for (size_t i = 0; i < hd; ++i) s += x[i] * x[i];
    float inv = 1.0f / std::sqrt(s / float(hd) + eps);
    for (size_t i = 0; i < hd; ++i)
      out[h * hd + i] = x[i] * inv * w[i] * silu(gate[h * hd + i]);
  }
}

// qwen35.rs:93-130 — depthwise causal conv step, state updated in place.
void causal_conv1d_step(const float* in, float* state, const float* w, size_t channels,
                        size_t k, float* out) {
  for (size_t c = 0; c < channels; ++c) {
    size_t sb = c * (k - 1), wb = c * k;
    float v = in[c] * w[wb + k - 1];
    for (size_t t = 0; t + 1 < k; ++t) v += state[sb + t] * w[wb + t];
    out[c] = v / (1.0f + std::exp(-v));
    for (size_t t = 0; t + 2 < k; ++t) state[sb + t] = state[sb + t + 1];
    state[sb + k - 2] = in[c];
  }
}

// qwen35.rs:163-225 — one Gated DeltaNet recurrent step, state [h][key][value].
void gdn_step(float* S, const float* q, const float* k, const float* v, const float* g,
              const float* beta, size_t heads, size_t kd, size_t vd, float* out) {
  std::vector<float> mem(vd), delta(vd);
  for (size_t h = 0; h < heads; ++h) {
    float* s = S + h * kd * vd;
    const float* kk = k + h * kd;
    const float* qq = q + h * kd;
    float decay = std::exp(g[h]);
    for (size_t i = 0; i < kd * vd; ++i) s[i] *= decay;
    std::fill(mem.begin(), mem.end(), 0.0f);
    for (size_t i = 0; i < kd; ++i)
      for (size_t j = 0; j < vd; ++j) mem[j] += s[i * vd + j] * kk[i];
    for (size_t j = 0; j < vd; ++j) delta[j] = (v[h * vd + j] - mem[j]) * beta[h];
    for (size_t i = 0; i < kd; ++i)
      for (size_t j = 0; j < vd; ++j) s[i * vd + j] += kk[i] * delta[j];
    for (size_t j = 0; j < vd; ++j) {
      float r = 0.0f;
      for (size_t i = 0; i < kd; ++i) r += s[i * vd + j] * qq[i];
      out[h * vd + j] = r;
    }
  }
}

// qwen35_runtime.rs:340-357
void l2_normalize_heads(float* v, size_t heads, size_t hd) {
  for (size_t h = 0; h < heads; ++h) {
    float s = 0.0f;
    for (size_t i = 0; i < hd; ++i) s += v[h * hd + i] * v[h * hd + i];
    float inv = 1.0f / std::sqrt(s + 1.0e-6f);
    for (size_t i = 0; i < hd; ++i) v[h * hd + i] *= inv;
  }
}

// metal.rs:1655-1679 — adjacent-pair RoPE; freq = theta^(-(2i)/d).
void rope(const float* in, size_t heads, size_t hd, size_t pos, float theta, float* out) {
  size_t pairs = hd / 2;
  for (size_t h = 0; h < heads; ++h)
    for (size_t p = 0; p < pairs; ++p) {
      float e = (2.0f * float(p)) / float(hd);
      float angle = float(pos) * std::pow(theta, -e);
      float sn = std::sin(angle), cs = std::cos(angle);
      size_t o = h * hd + p * 2;
      float a = in[o], b = in[o + 1];
      out[o] = a * cs - b * sn;
      out[o + 1] = a * sn + b * cs;
    }
}

// qwen35_runtime.rs:378-406 — RoPE on the first rotary_dim dims of each head.
void partial_rope(float* x, size_t heads, size_t hd, size_t rd, size_t pos, float theta) {
  std::vector<float> rot(heads * rd), outv(heads * rd);
  for (size_t h = 0; h < heads; ++h)
    std::memcpy(&rot[h * rd], x + h * hd, rd * 4);
  rope(rot.data(), heads, rd, pos, theta, outv.data());
  for (size_t h = 0; h < heads; ++h) std::memcpy(x + h * hd, &outv[h * rd], rd * 4);
}

float bf16_to_f32(uint16_t b) {
  uint32_t u = uint32_t(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}

// metal.rs:1681-1766 — GQA decode over a head-major cache [kvh][cap][hd]
// plus the current token's K/V from separate buffers. Cache element type is
// f32 (reference) or bf16 (this backend's device cache).
template <typename LoadK>
void attention_decode(const float* q, LoadK cache, const float* nk, const float* nv,
                      size_t qh, size_t kvh, size_t hd, size_t cached, size_t cap,
                      float* out) {
  float scale = 1.0f / std::sqrt(float(hd));
  size_t group = qh / kvh;
  size_t total = cached + 1;
  std::vector<float> scores(total);
  for (size_t h = 0; h < qh; ++h) {
    size_t kv = h / group;
    const float* qq = q + h * hd;
    float mx = -INFINITY;
    for (size_t t = 0; t < total; ++t) {
      float s = 0.0f;
      for (size_t d = 0; d < hd; ++d) {
        float kvv = t < cached ? cache(0, (kv * cap + t) * hd + d) : nk[kv * hd + d];
        s += qq[d] * kvv;
      }
      scores[t] = s;
      mx = std::max(mx, s * scale);
    }
    float norm = 0.0f;
    for (size_t t = 0; t < total; ++t) norm += std::exp(scores[t] * scale - mx);
    for (size_t d = 0; d < hd; ++d) {
      float r = 0.0f;
      for (size_t t = 0; t < total; ++t) {
        float wgt = std::exp(scores[t] * scale - mx) / norm;
        float vv = t < cached ? cache(1, (kv * cap + t) * hd + d) : nv[kv * hd + d];
        r += wgt * vv;
      }
      out[h * hd + d] = r;
    }
  }
}

// runtime.rs:4301-4309 — greedy argmax over finite logits, total order; among
// equal maxima `max_by` keeps the last index.
long argmax_last(const float* v, size_t n) {
  long best = -1;
  float bv = 0.0f;
  auto key = [](float f) {
    int32_t i;
    std::memcpy(&i, &f, 4);
    return i ^ int32_t(uint32_t(i >> 31) >> 1);  // f32::total_cmp ordering key
  };
  for (size_t i = 0; i < n; ++i) {
    if (!std::isfinite(v[i])) continue;
    if (best < 0 || key(v[i]) >= key(bv)) {
      best = long(i);
      bv = v[i];
    }
  }
  return best;
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI of the oracle (ctypes from tests/ and bench.py).
// ---------------------------------------------------------------------------
extern "C" {

int or_dequantize(uint32_t type, const uint8_t* bytes, size_t nbytes, size_t elements,
                  float* out) {
  int bb = block_bytes(type);
  if (bb == 0 || type == SI_GGML_TYPE_F32) return -1;
  if (elements == 0 || elements % kQK != 0) return -2;  // quant.rs:19-23
  if (nbytes != elements / kQK * size_t(bb)) return -3;  // quant.rs:28-33
  for (size_t b = 0; b < elements / kQK; ++b) deq_block(type, bytes + b * bb, out + b * kQK);
  return 0;
}

int or_matvec(uint32_t type, const uint8_t* w, size_t rows, size_t cols, const float* x,
              float* y, int threads) {
  if (block_bytes(type) == 0 || rows == 0 || cols == 0 ||
      (type != SI_GGML_TYPE_F32 && cols % kQK != 0))
    return -1;
  matvec(type, w, rows, cols, x, y, threads > 0 ? threads : omp_get_max_threads());
  return 0;
}

// Reference expectation of metal.rs:7498-7540: SiLU(gate.x) * (up.x).
int or_fused_gate_up(const uint8_t* gate, const uint8_t* up, size_t rows, size_t cols,
                     const float* x, float* out, int threads) {
  std::vector<float> g(rows), u(rows);
  int t = threads > 0 ? threads : omp_get_max_threads();
  matvec(SI_GGML_TYPE_Q4_K, gate, rows, cols, x, g.data(), t);
  matvec(SI_GGML_TYPE_Q4_K, up, rows, cols, x, u.data(), t);
  for (size_t r = 0; r < rows; ++r) out[r] = g[r] / (1.0f + std::exp(-g[r])) * u[r];
  return 0;
}

// metal.rs:3569-3732 / qwen35_runtime.rs:1447-1487 — down(SiLU(g)*u).
int or_fused_mlp(uint32_t gate_type, const uint8_t* gate, const uint8_t* up,
                 uint32_t down_type, const uint8_t* down, size_t inter, size_t hidden,
                 const float* x, float* y, int threads) {
  std::vector<float> act(inter);
  int t = threads > 0 ? threads : omp_get_max_threads();
  std::vector<float> g(inter), u(inter);
  matvec(gate_type, gate, inter, hidden, x, g.data(), t);
  matvec(gate_type, up, inter, hidden, x, u.data(), t);
  for (size_t r = 0; r < inter; ++r) act[r] = g[r] / (1.0f + std::exp(-g[r])) * u[r];
  matvec(down_type, down, hidden, inter, act.data(), y, t);
  return 0;
}

int or_rms_norm_heads(const float* in, const float* w, size_t heads, size_t hd, float eps,
                      float* out) {
  if (heads == 0 || hd == 0 || !(eps > 0.0f) || !std::isfinite(eps)) return -1;
  rms_norm_heads(in, w, heads, hd, eps, out);
  return 0;
}

int or_gated_rms_norm(const float* in, const float* gate, const float* w, size_t heads,
                      size_t hd, float eps, float* out) {
  if (heads == 0 || hd == 0 || !(eps > 0.0f) || !std::isfinite(eps)) return -1;
  gated_rms_norm(in, gate, w, heads, hd, eps, out);
  return 0;
}

int or_causal_conv1d_step(const float* in, float* state, const float* w, size_t channels,
                          size_t k, float* out) {
  if (channels == 0 || k < 2) return -1;
  causal_conv1d_step(in, state, w, channels, k, out);
  return 0;
}

int or_gdn_step(float* state, const float* q, const float* k, const float* v, const float* g,
                const float* beta, size_t heads, size_t kd, size_t vd, float* out) {
  if (heads == 0 || kd == 0 || vd == 0) return -1;
  gdn_step(state, q, k, v, g, beta, heads, kd, vd, out);
  return 0;
}

int or_rope(const float* in, size_t heads, size_t hd, size_t pos, float theta, float* out) {
  if (heads == 0 || hd == 0 || hd % 2) return -1;
  rope(in, heads, hd, pos, theta, out);
  return 0;
}

// cache_type: 0 = f32 caches, 1 = bf16 caches (uint16 bits).
int or_attention_decode(const float* q, const void* kc, const void* vc, int cache_type,
                        const float* nk, const float* nv, size_t qh, size_t kvh, size_t hd,
                        size_t cached, size_t cap, float* out) {
  if (qh == 0 || kvh == 0 || hd == 0 || qh % kvh || cached > cap) return -1;
  if (cache_type == 0) {
    const float* K = static_cast<const float*>(kc);
    const float* V = static_cast<const float*>(vc);
    attention_decode(q, [&](int which, size_t i) { return which ? V[i] : K[i]; }, nk, nv, qh,
                     kvh, hd, cached, cap, out);
  } else {
    const uint16_t* K = static_cast<const uint16_t*>(kc);
    const uint16_t* V = static_cast<const uint16_t*>(vc);
    attention_decode(
        q, [&](int which, size_t i) { return bf16_to_f32(which ? V[i] : K[i]); }, nk, nv, qh,
        kvh, hd, cached, cap, out);
  }
  return 0;
}

long or_argmax(const float* v, size_t n) { return argmax_last(v, n); }

uint16_t or_f32_to_bf16(float f) { return f32_to_bf16(f); }

// ---------------------------------------------------------------------------
// Layer- and model-level restatement (qwen35_runtime.rs). Weights are host
// pointers provided by the caller (the backend's synthetic model exposes its
// pinned host copy); the oracle never generates data itself.
// ---------------------------------------------------------------------------

struct or_tensor {
  const uint8_t* p;
  uint32_t type;
};

// qwen35_runtime.rs:409-624 with the gates supplied directly (config 3) when
// `gates` is non-null ([g[heads], beta[heads]]), otherwise computed from the
// F32 alpha/beta projections, A_log and dt_bias (qwen35_runtime.rs:593-601).
static void gdn_mixer(const si_model_config& c, const or_tensor* t, const float* x,
                      float* conv_state, float* rec_state, const float* gates, float* out,
                      int threads) {
  size_t H = c.hidden, kh = c.gdn_key_heads, vh = c.gdn_value_heads, d = c.gdn_head_dim;
  size_t kw = kh * d, vw = vh * d, proj = 2 * kw + vw;
  std::vector<float> qkv(proj), z(vw), mixed(proj);
  matvec(t[SI_T_SSM_QKV].type, t[SI_T_SSM_QKV].p, proj, H, x, qkv.data(), threads);
  matvec(t[SI_T_SSM_Z].type, t[SI_T_SSM_Z].p, vw, H, x, z.data(), threads);
  std::vector<float> g(vh), beta(vh);
  if (gates) {
    std::memcpy(g.data(), gates, vh * 4);
    std::memcpy(beta.data(), gates + vh, vh * 4);
  } else {
    std::vector<float> alpha(vh), bl(vh);
    matvec(SI_GGML_TYPE_F32, t[SI_T_SSM_ALPHA].p, vh, H, x, alpha.data(), threads);
    matvec(SI_GGML_TYPE_F32, t[SI_T_SSM_BETA].p, vh, H, x, bl.data(), threads);
    const float* alog = reinterpret_cast<const float*>(t[SI_T_SSM_A].p);
    const float* dt = reinterpret_cast<const float*>(t[SI_T_SSM_DT].p);
    for (size_t h = 0; h < vh; ++h) {
      beta[h] = 1.0f / (1.0f + std::exp(-bl[h]));
      g[h] = -std::exp(alog[h]) * softplus(alpha[h] + dt[h]);
    }
  }
  causal_conv1d_step(qkv.data(), conv_state, reinterpret_cast<const float*>(t[SI_T_SSM_CONV].p),
                     proj, c.conv_kernel, mixed.data());
  std::vector<float> qn(mixed.begin(), mixed.begin() + kw);
  std::vector<float> kn(mixed.begin() + kw, mixed.begin() + 2 * kw);
  l2_normalize_heads(qn.data(), kh, d);
  l2_normalize_heads(kn.data(), kh, d);
  size_t rep = vh / kh;
  std::vector<float> q(vw), k(vw);
  float sq = std::sqrt(float(d));
  for (size_t h = 0; h < vh; ++h)
    for (size_t i = 0; i < d; ++i) {
      q[h * d + i] = qn[(h / rep) * d + i] / sq;
      k[h * d + i] = kn[(h / rep) * d + i];
    }
  std::vector<float> core(vw), normed(vw);
  gdn_step(rec_state, q.data(), k.data(), mixed.data() + 2 * kw, g.data(), beta.data(), vh, d, d,
           core.data());
  gated_rms_norm(core.data(), z.data(), reinterpret_cast<const float*>(t[SI_T_SSM_NORM].p), vh,
                 d, c.rms_eps, normed.data());
  matvec(t[SI_T_SSM_OUT].type, t[SI_T_SSM_OUT].p, H, vw, normed.data(), out, threads);
}

// qwen35_runtime.rs:628-867 with the head-major cache of cache.rs:1-4.
static void attention_mixer(const si_model_config& c, const or_tensor* t, const float* x,
                            size_t position, uint16_t* kc, uint16_t* vc, size_t* cached,
                            float* out, int threads) {
  size_t H = c.hidden, qh = c.attn_q_heads, kvh = c.attn_kv_heads, hd = c.attn_head_dim;
  size_t qw = qh * hd, kvw = kvh * hd, cap = c.kv_capacity;
  std::vector<float> qg(2 * qw), k(kvw), v(kvw);
  matvec(t[SI_T_ATTN_Q].type, t[SI_T_ATTN_Q].p, 2 * qw, H, x, qg.data(), threads);
  matvec(t[SI_T_ATTN_K].type, t[SI_T_ATTN_K].p, kvw, H, x, k.data(), threads);
  matvec(t[SI_T_ATTN_V].type, t[SI_T_ATTN_V].p, kvw, H, x, v.data(), threads);
  std::vector<float> q(qw), kk(kvw);
  rms_norm_heads(qg.data(), reinterpret_cast<const float*>(t[SI_T_ATTN_QNORM].p), qh, hd,
                 c.rms_eps, q.data());
  rms_norm_heads(k.data(), reinterpret_cast<const float*>(t[SI_T_ATTN_KNORM].p), kvh, hd,
                 c.rms_eps, kk.data());
  partial_rope(q.data(), qh, hd, c.rotary_dim, position, c.rope_theta);
  partial_rope(kk.data(), kvh, hd, c.rotary_dim, position, c.rope_theta);
  std::vector<float> att(qw);
  attention_decode(
      q.data(), [&](int which, size_t i) { return bf16_to_f32(which ? vc[i] : kc[i]); },
      kk.data(), v.data(), qh, kvh, hd, *cached, cap, att.data());
  for (size_t h = 0; h < kvh; ++h)
    for (size_t i = 0; i < hd; ++i) {
      kc[(h * cap + *cached) * hd + i] = f32_to_bf16(kk[h * hd + i]);
      vc[(h * cap + *cached) * hd + i] = f32_to_bf16(v[h * hd + i]);
    }
  *cached += 1;
  for (size_t i = 0; i < qw; ++i) att[i] = att[i] / (1.0f + std::exp(-qg[qw + i]));
  matvec(t[SI_T_ATTN_O].type, t[SI_T_ATTN_O].p, H, qw, att.data(), out, threads);
}

struct or_model {
  si_model_config c;
  std::vector<std::vector<or_tensor>> t;  // [layers + 1][SI_T_COUNT]
  std::vector<std::vector<float>> conv, rec;
  std::vector<std::vector<uint16_t>> kc, vc;
  std::vector<size_t> cached;
  int threads;
};

or_model* or_model_create(const si_model_config* c, const void* const* ptrs,
                          const uint32_t* types, int threads) {
  auto* m = new or_model();
  m->c = *c;
  m->threads = threads > 0 ? threads : omp_get_max_threads();
  m->t.resize(c->layers + 1, std::vector<or_tensor>(SI_T_COUNT));
  for (uint32_t l = 0; l <= c->layers; ++l)
    for (int i = 0; i < SI_T_COUNT; ++i) {
      m->t[l][i].p = static_cast<const uint8_t*>(ptrs[size_t(l) * SI_T_COUNT + i]);
      m->t[l][i].type = types[size_t(l) * SI_T_COUNT + i];
    }
  size_t proj = (2 * c->gdn_key_heads + c->gdn_value_heads) * c->gdn_head_dim;
  m->conv.resize(c->layers);
  m->rec.resize(c->layers);
  m->kc.resize(c->layers);
  m->vc.resize(c->layers);
  m->cached.assign(c->layers, 0);
  for (uint32_t l = 0; l < c->layers; ++l) {
    if ((l + 1) % c->attn_interval != 0) {
      m->conv[l].assign(proj * (c->conv_kernel - 1), 0.0f);
      m->rec[l].assign(size_t(c->gdn_value_heads) * c->gdn_head_dim * c->gdn_head_dim, 0.0f);
    } else {
      size_t n = size_t(c->attn_kv_heads) * c->kv_capacity * c->attn_head_dim;
      m->kc[l].assign(n, 0);
      m->vc[l].assign(n, 0);
    }
  }
  return m;
}

void or_model_destroy(or_model* m) { delete m; }

// qwen35_runtime.rs:1329-1490 — one decoder block, hidden updated in place.
static int decoder_block(or_model* m, uint32_t l, size_t position, float* hidden) {
  const si_model_config& c = m->c;
  const or_tensor* t = m->t[l].data();
  size_t H = c.hidden, I = c.intermediate;
  std::vector<float> normed(H), mix(H);
  rms_norm_heads(hidden, reinterpret_cast<const float*>(t[SI_T_ATTN_NORM].p), 1, H, c.rms_eps,
                 normed.data());
  if ((l + 1) % c.attn_interval != 0) {
    gdn_mixer(c, t, normed.data(), m->conv[l].data(), m->rec[l].data(), nullptr, mix.data(),
              m->threads);
  } else {
    if (m->cached[l] >= c.kv_capacity) return -2;
    attention_mixer(c, t, normed.data(), position, m->kc[l].data(), m->vc[l].data(),
                    &m->cached[l], mix.data(), m->threads);
  }
  for (size_t i = 0; i < H; ++i) hidden[i] += mix[i];
  rms_norm_heads(hidden, reinterpret_cast<const float*>(t[SI_T_POST_NORM].p), 1, H, c.rms_eps,
                 normed.data());
  std::vector<float> g(I), u(I), act(I), y(H);
  matvec(t[SI_T_FFN_GATE].type, t[SI_T_FFN_GATE].p, I, H, normed.data(), g.data(), m->threads);
  matvec(t[SI_T_FFN_UP].type, t[SI_T_FFN_UP].p, I, H, normed.data(), u.data(), m->threads);
  for (size_t r = 0; r < I; ++r) act[r] = g[r] / (1.0f + std::exp(-g[r])) * u[r];
  matvec(t[SI_T_FFN_DOWN].type, t[SI_T_FFN_DOWN].p, H, I, act.data(), y.data(), m->threads);
  for (size_t i = 0; i < H; ++i) hidden[i] += y[i];
  return 0;
}

// qwen35_runtime.rs:2122-2130 — embedding row dequant.
int or_model_embed(or_model* m, uint32_t token, float* out) {
  const si_model_config& c = m->c;
  if (token >= c.vocab) return -1;
  const or_tensor& e = m->t[c.layers][SI_T_TOKEN_EMBD];
  deq_row(e.type, e.p + size_t(token) * row_bytes(e.type, c.hidden), c.hidden, out);
  return 0;
}

// qwen35_runtime.rs:1776-1941 (sequential semantics of the layer loop).
int or_model_decode_hidden(or_model* m, size_t position, float* hidden) {
  for (uint32_t l = 0; l < m->c.layers; ++l) {
    int rc = decoder_block(m, l, position, hidden);
    if (rc) return rc;
  }
  return 0;
}

// qwen35_runtime.rs:2132-2192 — output_norm (1+w) then the output head.
int or_model_logits(or_model* m, const float* hidden, float* logits) {
  const si_model_config& c = m->c;
  std::vector<float> normed(c.hidden);
  rms_norm_heads(hidden, reinterpret_cast<const float*>(m->t[c.layers][SI_T_OUTPUT_NORM].p), 1,
                 c.hidden, c.rms_eps, normed.data());
  const or_tensor& o = m->t[c.layers][SI_T_OUTPUT];
  matvec(o.type, o.p, c.vocab, c.hidden, normed.data(), logits, m->threads);
  return 0;
}

// runtime.rs:3560-3614 — token-by-token prefill, then greedy decode with
// runtime::argmax. Returns the number of generated ids written to `out`.
long or_model_generate(or_model* m, const uint32_t* prompt, size_t n_prompt, size_t max_new,
                       uint32_t* out) {
  const si_model_config& c = m->c;
  std::vector<float> hidden(c.hidden), logits(c.vocab);
  for (size_t p = 0; p < n_prompt; ++p) {
    if (or_model_embed(m, prompt[p], hidden.data())) return -1;
    if (or_model_decode_hidden(m, p, hidden.data())) return -2;
  }
  or_model_logits(m, hidden.data(), logits.data());
  size_t n = 0;
  for (size_t i = 0; i < max_new; ++i) {
    long tok = argmax_last(logits.data(), c.vocab);
    if (tok < 0) return -3;
    out[n++] = uint32_t(tok);
    if (uint32_t(tok) == c.eos_token) break;
    if (or_model_embed(m, uint32_t(tok), hidden.data())) return -1;
    if (or_model_decode_hidden(m, n_prompt + i, hidden.data())) return -2;
    or_model_logits(m, hidden.data(), logits.data());
  }
  return long(n);
}

// Standalone Gated DeltaNet layer (config 3): qkv/z projections, conv,
// normalisation, recurrence, gated norm and ssm_out, gates supplied directly.
int or_gdn_layer(const si_model_config* c, const void* const* ptrs, const uint32_t* types,
                 const float* x, float* conv_state, float* rec_state, const float* gates,
                 float* out, int threads) {
  std::vector<or_tensor> t(SI_T_COUNT);
  for (int i = 0; i < SI_T_COUNT; ++i) {
    t[i].p = static_cast<const uint8_t*>(ptrs[i]);
    t[i].type = types[i];
  }
  gdn_mixer(*c, t.data(), x, conv_state, rec_state, gates, out,
            threads > 0 ? threads : omp_get_max_threads());
  return 0;
}

// Standalone full-attention mixer (config 4) over a bf16 head-major cache.
int or_attention_layer(const si_model_config* c, const void* const* ptrs, const uint32_t* types,
                       const float* x, size_t position, uint16_t* kc, uint16_t* vc,
                       size_t* cached, float* out, int threads) {
  std::vector<or_tensor> t(SI_T_COUNT);
  for (int i = 0; i < SI_T_COUNT; ++i) {
    t[i].p = static_cast<const uint8_t*>(ptrs[i]);
    t[i].type = types[i];
  }
  if (*cached >= c->kv_capacity) return -2;
  attention_mixer(*c, t.data(), x, position, kc, vc, cached, out,
                  threads > 0 ? threads : omp_get_max_threads());
  return 0;
}

}  // extern "C"
