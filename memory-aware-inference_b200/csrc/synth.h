// Seeded synthetic GGUF-shaped weights (counter-based, so any shard of a
// tensor can be generated independently and matches the full tensor).
//
// Stream: SplitMix64 over a counter. For tensor key K, 64-bit word i of the
// tensor's byte stream is splitmix64(K + i * golden). Quant and scale bytes
// are those bytes (uniform 0..255); the fp16 d / dmin fields of every
// super-block are |N(0, 0.02)| rounded to nearest-even, drawn by Box-Muller
// from the counter stream of key K ^ kScaleSalt at the block index. F32
// tensors are N(mean, std) per element from key K at the element index.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

namespace si {

inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kScaleSalt = 0xD1B54A32D192ED03ull;

inline uint64_t tensor_key(uint64_t seed, uint32_t layer, uint32_t tensor) {
  return splitmix64(seed ^ splitmix64((uint64_t(layer) << 8) | tensor));
}

inline double uniform01(uint64_t u) { return (double((u >> 11) + 1)) * (1.0 / 9007199254740993.0); }

// Standard normal from counter `i` of key `k` (Box-Muller, cosine branch).
inline double gauss(uint64_t k, uint64_t i) {
  const double u1 = uniform01(splitmix64(k + (2 * i) * kGolden));
  const double u2 = uniform01(splitmix64(k + (2 * i + 1) * kGolden));
  return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

// IEEE binary32 -> binary16, round to nearest even (finite inputs).
inline uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int32_t exp = int32_t((x >> 23) & 0xff) - 127 + 15;
  uint32_t mant = x & 0x7fffffu;
  if (((x >> 23) & 0xff) == 0xff) return uint16_t(sign | 0x7c00u | (mant ? 0x200u : 0));
  if (exp >= 31) return uint16_t(sign | 0x7c00u);
  if (exp <= 0) {
    if (exp < -10) return uint16_t(sign);
    mant |= 0x800000u;
    const uint32_t shift = uint32_t(14 - exp);
    uint32_t h = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1))) ++h;
    return uint16_t(sign | h);
  }
  uint32_t h = (uint32_t(exp) << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
  return uint16_t(sign | h);
}

// Bytes [off, off + n) of a quantized tensor's stream with key `k`; block
// headers are NOT patched here (see patch_scales).
inline void fill_bytes(uint64_t k, uint64_t off, uint64_t n, uint8_t* dst) {
  uint64_t i = off;
  const uint64_t end = off + n;
  while (i < end) {
    const uint64_t w = splitmix64(k + (i >> 3) * kGolden);
    const uint32_t b0 = uint32_t(i & 7);
    for (uint32_t b = b0; b < 8 && i < end; ++b, ++i) *dst++ = uint8_t(w >> (8 * b));
  }
}

// Overwrite the fp16 scale fields of global super-block `block` at `dst`.
inline void patch_scales(uint64_t k, uint32_t type, uint64_t block, uint8_t* dst) {
  const uint64_t ks = k ^ kScaleSalt;
  const uint16_t d = f32_to_f16(float(std::fabs(0.02 * gauss(ks, 2 * block))));
  if (type == 14u) {  // Q6_K: d at bytes 208..209
    dst[208] = uint8_t(d);
    dst[209] = uint8_t(d >> 8);
    return;
  }
  const uint16_t dm = f32_to_f16(float(std::fabs(0.02 * gauss(ks, 2 * block + 1))));
  dst[0] = uint8_t(d);
  dst[1] = uint8_t(d >> 8);
  dst[2] = uint8_t(dm);
  dst[3] = uint8_t(dm >> 8);
}

// Centered K-quant scales: every sub-block gets a scale in 0..8 and a min
// ~ offset * scale with dmin = d (offset 7.5 for Q4_K, 15.5 for Q5_K), so the
// dequantised row is roughly zero-mean, as in real quantised weights. The 12
// packed bytes follow the 6-bit layout that get_scale_min reads.
inline void center_scales(uint64_t k, uint32_t type, uint64_t block, uint8_t* dst) {
  const uint64_t r = splitmix64((k ^ 0xA5A5A5A5A5A5A5A5ull) + block * kGolden);
  uint8_t sc[8], mn[8];
  const double off = type == 13u ? 15.5 : 7.5;
  const int smax = type == 13u ? 4 : 8;
  for (int j = 0; j < 8; ++j) {
    sc[j] = uint8_t(((r >> (8 * j)) & 0xff) % uint64_t(smax + 1));
    const long m = std::lround(off * sc[j]);
    mn[j] = uint8_t(m > 63 ? 63 : m);
  }
  uint8_t* s = dst + 4;
  for (int j = 0; j < 4; ++j) {
    s[j] = uint8_t((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = uint8_t((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    s[j + 8] = uint8_t((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
  }
  dst[2] = dst[0];  // dmin = d
  dst[3] = dst[1];
}

}  // namespace si
