// Batch-1 GGUF K-quant matvec for sm_100a.
//
// Replaces the Metal kernels si_q4_k_matvec / si_q5_k_matvec / si_q6_k_matvec
// (+ their rows4 variants), si_q4_k_fused_gate_up and the grouped matvec
// (src/metal.rs:310-494, 498-587, 770-1050, 4532-4780 in the reference).
//
// Design (one CTA per SM, persistent over a contiguous range of rows):
//  * A producer warp streams whole rows (2,880 B for a Q4_K 5120-column row)
//    from HBM into a ring of shared-memory slots with non-tensor bulk async
//    copies (cp.async.bulk, L2 evict_first), tracked by full/empty mbarriers.
//  * 16 consumer warps = 32 teams of 16 lanes; a team owns one row at a time.
//    Lane l of a team always decodes the same 64-element unit of each
//    super-block (Q4_K/Q5_K: group l%4; Q6_K: half/16-run l%4), so the 6-bit
//    scale/min extraction pattern is fixed per lane and never diverges.
//  * Weights are decoded in registers: each 4/5/6-bit quant q becomes the
//    float 1 + q/2^k by placing its bits in the mantissa (LOP3 + PRMT, no
//    int->float conversion), multiplied with x by packed fp32 FMA
//    (fma.rn.f32x2), and the offset is removed per sub-block with the
//    precomputed sub-block sums of x: sum(q x) = 2^k (A - X).
//  * The input vector x (and an optional fused RMSNorm / gated-norm /
//    sigmoid-gate transform of it) lives in shared memory, with its 16- and
//    32-element partial sums. Epilogues: store, residual add, SwiGLU pair.
//  * Accumulation is fp32 throughout; team results are combined with
//    warp shuffles. Tensor cores are not used: batch-1 is not a contraction.
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "qmatvec.cuh"

namespace si {

constexpr int kConsumerWarps = 16;
constexpr int kThreads = kConsumerWarps * 32 + 32;
constexpr int kTeams = kConsumerWarps * 2;
constexpr int kTeamLanes = 16;
constexpr int kMaxSlots = 64;
constexpr uint32_t kMaxDynSmem = 227 * 1024;

__device__ __forceinline__ float mant_float(uint32_t word, int j) {
  // byte j of `word` becomes bits 16..23 of a float whose top byte is 0x3F.
  return as_f(__byte_perm(word, 0x3F000000u, 0x7044u | (uint32_t(j) << 8)));
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// 16 bytes from a 2-byte-aligned shared-memory address.
__device__ __forceinline__ uint4 lds16_a2(const uint8_t* p) {
  uint32_t off = smem_u32(p) & 3u;
  const uint32_t* w = reinterpret_cast<const uint32_t*>(p - off);
  uint32_t a = w[0], b = w[1], c = w[2], d = w[3], e = w[4];
  uint32_t sh = off * 8u;
  return make_uint4(__funnelshift_r(a, b, sh), __funnelshift_r(b, c, sh),
                    __funnelshift_r(c, d, sh), __funnelshift_r(d, e, sh));
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// ---------------------------------------------------------------------------
// Q4_K: 144-byte blocks [d f16][dmin f16][12 B scales][128 B quants]. Unit g
// (0..3) of a block covers quant bytes 32g..32g+31: low nibbles are elements
// 64g+0..31 (scale index 2g), high nibbles 64g+32..63 (scale index 2g+1).
// ---------------------------------------------------------------------------
struct Q4KUnitScales {
  float d1, m1, d2, m2;
};

__device__ __forceinline__ Q4KUnitScales q4k_scales(const uint4& hdr, int g) {
  const uint32_t W1 = hdr.y, W2 = hdr.z, W3 = hdr.w;
  const uint32_t sh = 16u * uint32_t(g & 1);
  uint32_t sa, ma, sb, mb;
  if (g < 2) {
    sa = (W1 >> sh) & 63u;
    sb = (W1 >> (sh + 8)) & 63u;
    ma = (W2 >> sh) & 63u;
    mb = (W2 >> (sh + 8)) & 63u;
  } else {
    sa = ((W3 >> sh) & 15u) | (((W1 >> (sh + 6)) & 3u) << 4);
    sb = ((W3 >> (sh + 8)) & 15u) | (((W1 >> (sh + 14)) & 3u) << 4);
    ma = ((W3 >> (sh + 4)) & 15u) | (((W2 >> (sh + 6)) & 3u) << 4);
    mb = ((W3 >> (sh + 12)) & 15u) | (((W2 >> (sh + 14)) & 3u) << 4);
  }
  const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hdr.x));
  Q4KUnitScales s;
  s.d1 = dm.x * float(sa);
  s.m1 = dm.y * float(ma);
  s.d2 = dm.x * float(sb);
  s.m2 = dm.y * float(mb);
  return s;
}

// A_lo / A_hi for one Q4_K or Q5_K unit: sums of (1 + q/2^k) * x.
template <int KIND>
__device__ __forceinline__ void unit_sums_q45(const uint4 qa, const uint4 qb, const uint4 ha,
                                              const uint4 hb, int g, const float* xp,
                                              float& alo, float& ahi) {
  float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t w = word_of(k < 4 ? qa : qb, k & 3);
    uint32_t vl, vh;
    if (KIND == 4) {
      // q in mantissa bits 19..22 -> 1 + q/16
      vl = ((w << 3) & 0x78787878u) | 0x80808080u;
      vh = ((w >> 1) & 0x78787878u) | 0x80808080u;
    } else {
      // Q5_K: q5 = nibble + 16*bit(qh, 2g / 2g+1), placed at bits 18..22 -> 1 + q/32
      const uint32_t h = word_of(k < 4 ? ha : hb, k & 3);
      const uint32_t bl = (h >> (2 * g)) & 0x01010101u;
      const uint32_t bh = (h >> (2 * g + 1)) & 0x01010101u;
      vl = (((w & 0x0F0F0F0Fu) | (bl << 4)) << 2) | 0x80808080u;
      vh = ((((w >> 4) & 0x0F0F0F0Fu) | (bh << 4)) << 2) | 0x80808080u;
    }
    const float4 xl = *reinterpret_cast<const float4*>(xp + 4 * k);
    const float4 xh = *reinterpret_cast<const float4*>(xp + 32 + 4 * k);
    lo = ffma2(make_float2(mant_float(vl, 0), mant_float(vl, 1)), make_float2(xl.x, xl.y), lo);
    lo = ffma2(make_float2(mant_float(vl, 2), mant_float(vl, 3)), make_float2(xl.z, xl.w), lo);
    hi = ffma2(make_float2(mant_float(vh, 0), mant_float(vh, 1)), make_float2(xh.x, xh.y), hi);
    hi = ffma2(make_float2(mant_float(vh, 2), mant_float(vh, 3)), make_float2(xh.z, xh.w), hi);
  }
  alo = lo.x + lo.y;
  ahi = hi.x + hi.y;
}

template <uint32_t TYPE>
struct RowDot;

template <>
struct RowDot<SI_GGML_TYPE_Q4_K> {
  static constexpr uint32_t BB = 144;
  template <int NR>
  __device__ __forceinline__ static void run(const uint8_t* const* rows, const float* xs,
                                             const float* xs32, uint32_t cols, int tl,
                                             float* acc) {
    const int g = tl & 3;
    const int nunits = int(cols >> 6);
    for (int u = tl; u < nunits; u += kTeamLanes) {
      const int b = u >> 2;
      const float* xp = xs + b * 256 + g * 64;
      const float Xl = xs32[b * 8 + g * 2], Xh = xs32[b * 8 + g * 2 + 1];
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        const uint8_t* blk = rows[r] + b * BB;
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
        const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * g);
        float alo, ahi;
        unit_sums_q45<4>(qa, qb, qa, qb, g, xp, alo, ahi);
        const Q4KUnitScales s = q4k_scales(hdr, g);
        acc[r] += s.d1 * (16.0f * (alo - Xl)) - s.m1 * Xl;
        acc[r] += s.d2 * (16.0f * (ahi - Xh)) - s.m2 * Xh;
      }
    }
  }
};

template <>
struct RowDot<SI_GGML_TYPE_Q5_K> {
  static constexpr uint32_t BB = 176;
  template <int NR>
  __device__ __forceinline__ static void run(const uint8_t* const* rows, const float* xs,
                                             const float* xs32, uint32_t cols, int tl,
                                             float* acc) {
    const int g = tl & 3;
    const int nunits = int(cols >> 6);
    for (int u = tl; u < nunits; u += kTeamLanes) {
      const int b = u >> 2;
      const float* xp = xs + b * 256 + g * 64;
      const float Xl = xs32[b * 8 + g * 2], Xh = xs32[b * 8 + g * 2 + 1];
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        const uint8_t* blk = rows[r] + b * BB;
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 ha = *reinterpret_cast<const uint4*>(blk + 16);
        const uint4 hb = *reinterpret_cast<const uint4*>(blk + 32);
        const uint4 qa = *reinterpret_cast<const uint4*>(blk + 48 + 32 * g);
        const uint4 qb = *reinterpret_cast<const uint4*>(blk + 64 + 32 * g);
        float alo, ahi;
        unit_sums_q45<5>(qa, qb, ha, hb, g, xp, alo, ahi);
        const Q4KUnitScales s = q4k_scales(hdr, g);
        acc[r] += s.d1 * (32.0f * (alo - Xl)) - s.m1 * Xl;
        acc[r] += s.d2 * (32.0f * (ahi - Xh)) - s.m2 * Xh;
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Q6_K: 210-byte blocks [ql 128][qh 64][int8 scales 16][d f16]. Unit ul (0..3)
// is half h = ul/2 and 16-run i0 = 16*(ul%2): q1..q4 of elements
// 128h + i0 + {0,32,64,96} + (0..15), scales 8h + ul%2 + {0,2,4,6}.
// ---------------------------------------------------------------------------
template <>
struct RowDot<SI_GGML_TYPE_Q6_K> {
  static constexpr uint32_t BB = 210;
  template <int NR>
  __device__ __forceinline__ static void run(const uint8_t* const* rows, const float* xs,
                                             const float* xs16, uint32_t cols, int tl,
                                             float* acc) {
    const int ul = tl & 3;
    const int h = ul >> 1, i0 = (ul & 1) * 16;
    const int nunits = int(cols >> 6);
    for (int u = tl; u < nunits; u += kTeamLanes) {
      const int b = u >> 2;
      const int e0 = b * 256 + 128 * h + i0;
      const float* xp = xs + e0;
      float X[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) X[m] = xs16[(e0 >> 4) + 2 * m];
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        const uint8_t* blk = rows[r] + b * BB;
        const uint4 L1 = lds16_a2(blk + 64 * h + i0);
        const uint4 L2 = lds16_a2(blk + 64 * h + 32 + i0);
        const uint4 H = lds16_a2(blk + 128 + 32 * h + i0);
        const uint8_t* scp = blk + 192 + 8 * h + (ul & 1);
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(blk + 208));
        float2 a[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) a[m] = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t l1 = word_of(L1, k), l2 = word_of(L2, k), hh = word_of(H, k);
          uint32_t v[4];
          v[0] = ((l1 << 1) & 0x1E1E1E1Eu) | ((hh << 5) & 0x60606060u) | 0x80808080u;
          v[1] = ((l2 << 1) & 0x1E1E1E1Eu) | ((hh << 3) & 0x60606060u) | 0x80808080u;
          v[2] = ((l1 >> 3) & 0x1E1E1E1Eu) | ((hh << 1) & 0x60606060u) | 0x80808080u;
          v[3] = ((l2 >> 3) & 0x1E1E1E1Eu) | ((hh >> 1) & 0x60606060u) | 0x80808080u;
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float4 xv = *reinterpret_cast<const float4*>(xp + 32 * m + 4 * k);
            a[m] = ffma2(make_float2(mant_float(v[m], 0), mant_float(v[m], 1)),
                         make_float2(xv.x, xv.y), a[m]);
            a[m] = ffma2(make_float2(mant_float(v[m], 2), mant_float(v[m], 3)),
                         make_float2(xv.z, xv.w), a[m]);
          }
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float sc = float(int(static_cast<int8_t>(scp[2 * m])));
          const float A = a[m].x + a[m].y;
          acc[r] += (d * sc) * (64.0f * (A - X[m]) - 32.0f * X[m]);
        }
      }
    }
  }
};

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
struct ItemSrc {
  const uint8_t* g;  // global address of the row
  float* y;
  const float* resid;
  uint32_t row;
};

__device__ __forceinline__ ItemSrc item_src(const QmvParams& p, uint32_t item, uint32_t rb,
                                            int which) {
  ItemSrc s;
  if (p.pair) {
    s.g = p.seg[which].w + size_t(item) * rb;
    s.y = p.seg[0].y;
    s.resid = p.seg[0].resid;
    s.row = item;
    return s;
  }
  uint32_t r = item;
  int k = 0;
#pragma unroll
  for (int i = 0; i < 3; ++i)
    if (k < int(p.nseg) - 1 && r >= p.seg[k].rows) {
      r -= p.seg[k].rows;
      ++k;
    }
  s.g = p.seg[k].w + size_t(r) * rb;
  s.y = p.seg[k].y;
  s.resid = p.seg[k].resid;
  s.row = r;
  return s;
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

template <uint32_t TYPE, int NR>
__global__ void __launch_bounds__(kThreads, 1)
    qmv_kernel(const __grid_constant__ QmvParams p, uint32_t slot_bytes, uint32_t nslots,
               uint32_t slots_off) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_abort;
  __shared__ float s_red[kConsumerWarps];

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + nslots;
  const uint32_t cols = p.cols;
  float* xs = reinterpret_cast<float*>(smem + 16 * nslots);
  float* xs16 = xs + cols;
  float* xs32 = xs16 + cols / 16;
  uint8_t* slots = smem + slots_off;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rb = cols / 256 * RowDot<TYPE>::BB;
  const uint32_t i0 = uint32_t(uint64_t(blockIdx.x) * p.items / gridDim.x);
  const uint32_t i1 = uint32_t(uint64_t(blockIdx.x + 1) * p.items / gridDim.x);
  const uint32_t n_items = i1 - i0;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < nslots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kConsumerWarps) {
    // ---------------- producer: one elected lane streams rows -------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t issued = 0;
      for (uint32_t k = 0; k < n_items; ++k) {
        const uint32_t s = k % nslots, n = k / nslots;
        if (n > 0 && !mbar_wait_bounded(&empty[s], (n - 1) & 1)) {
          atomicOr(p.err, KERR_TIMEOUT_EMPTY);
          s_abort = 1;
          break;
        }
        if (*reinterpret_cast<volatile int*>(&s_abort)) break;
        uint8_t* dst = slots + size_t(s) * slot_bytes;
        uint32_t tx = 0;
#pragma unroll
        for (int w = 0; w < NR; ++w) {
          const ItemSrc src = item_src(p, i0 + k, rb, w);
          const uintptr_t a = reinterpret_cast<uintptr_t>(src.g);
          const uintptr_t a0 = a & ~uintptr_t(15);
          const uintptr_t a1 = (a + rb + 15) & ~uintptr_t(15);
          tx += uint32_t(a1 - a0);
        }
        mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
        for (int w = 0; w < NR; ++w) {
          const ItemSrc src = item_src(p, i0 + k, rb, w);
          const uintptr_t a = reinterpret_cast<uintptr_t>(src.g);
          const uintptr_t a0 = a & ~uintptr_t(15);
          const uintptr_t a1 = (a + rb + 15) & ~uintptr_t(15);
          bulk_g2s(dst + w * (slot_bytes / NR), reinterpret_cast<const void*>(a0),
                   uint32_t(a1 - a0), &full[s], pol);
        }
        ++issued;
      }
      if (*reinterpret_cast<volatile int*>(&s_abort)) {
        // Drain: wait (bounded) until every copy this CTA issued has landed.
        const uint32_t first = issued > nslots ? issued - nslots : 0;
        for (uint32_t k = first; k < issued; ++k)
          if (!mbar_wait_bounded(&full[k % nslots], (k / nslots) & 1))
            atomicOr(p.err, KERR_TIMEOUT_DRAIN);
      }
    }
    return;
  }

  // ---------------- consumers: build x in shared memory -------------------
  pdl_wait();
  const int ct = threadIdx.x;  // 0 .. 511
  constexpr int NC = kConsumerWarps * 32;
  if (p.xmode == XM_RAW) {
    for (uint32_t i = ct * 4; i < cols; i += NC * 4)
      *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(p.x + i);
  } else if (p.xmode == XM_RMS1P) {
    float ss = 0.f;
    for (uint32_t i = ct; i < cols; i += NC) {
      const float v = p.x[i];
      xs[i] = v;
      ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    consumer_sync();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) tot += s_red[w];
    const float inv = 1.0f / sqrtf(tot / float(cols) + p.eps);
    for (uint32_t i = ct; i < cols; i += NC) xs[i] = xs[i] * inv * (1.0f + p.xw[i]);
  } else if (p.xmode == XM_GATED) {
    // One warp per head (head_dim a multiple of 32).
    const uint32_t hd = p.head_dim, heads = cols / hd;
    for (uint32_t h = warp; h < heads; h += kConsumerWarps) {
      float ss = 0.f;
      for (uint32_t i = lane; i < hd; i += 32) {
        const float v = p.x[h * hd + i];
        ss += v * v;
      }
      ss = warp_sum(ss);
      const float inv = 1.0f / sqrtf(ss / float(hd) + p.eps);
      for (uint32_t i = lane; i < hd; i += 32) {
        const float v = p.x[h * hd + i];
        const float z = p.xaux[h * hd + i];
        xs[h * hd + i] = v * inv * p.xw[i] * (z / (1.0f + expf(-z)));
      }
    }
  } else {  // XM_SIGGATE
    for (uint32_t i = ct; i < cols; i += NC) {
      const float gte = p.xaux[i];
      xs[i] = p.x[i] / (1.0f + expf(-gte));
    }
  }
  consumer_sync();
  for (uint32_t j = ct; j < cols / 16; j += NC) {
    const float4* q = reinterpret_cast<const float4*>(xs + 16 * j);
    float4 a = q[0], b = q[1], c = q[2], d = q[3];
    xs16[j] = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w)) +
              (((c.x + c.y) + (c.z + c.w)) + ((d.x + d.y) + (d.z + d.w)));
  }
  consumer_sync();
  for (uint32_t j = ct; j < cols / 32; j += NC) xs32[j] = xs16[2 * j] + xs16[2 * j + 1];
  consumer_sync();

  // ---------------- consumers: one row (pair) per team ---------------------
  const int team = ct >> 4, tl = ct & 15;
  const unsigned tmask = (lane < 16) ? 0x0000ffffu : 0xffff0000u;
  const float* xsum = (TYPE == SI_GGML_TYPE_Q6_K) ? xs16 : xs32;
  for (uint32_t k = team; k < n_items; k += kTeams) {
    const uint32_t s = k % nslots, n = k / nslots;
    if (!mbar_wait_bounded(&full[s], n & 1)) {
      atomicOr(p.err, KERR_TIMEOUT_FULL);
      s_abort = 1;
      break;
    }
    const uint8_t* base = slots + size_t(s) * slot_bytes;
    const uint8_t* rows[NR];
    ItemSrc src0 = item_src(p, i0 + k, rb, 0);
#pragma unroll
    for (int w = 0; w < NR; ++w) {
      const ItemSrc src = item_src(p, i0 + k, rb, w);
      rows[w] = base + w * (slot_bytes / NR) + (reinterpret_cast<uintptr_t>(src.g) & 15);
    }
    float acc[NR];
#pragma unroll
    for (int w = 0; w < NR; ++w) acc[w] = 0.f;
    RowDot<TYPE>::template run<NR>(rows, xs, xsum, cols, tl, acc);
#pragma unroll
    for (int w = 0; w < NR; ++w) {
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) acc[w] += __shfl_xor_sync(tmask, acc[w], o);
    }
    __syncwarp(tmask);
    if (tl == 0) {
      mbar_arrive(&empty[s]);
      float out;
      if (NR == 2) {
        const float g = acc[0];
        out = g / (1.0f + expf(-g)) * acc[NR - 1];
      } else {
        out = acc[0];
      }
      if (src0.resid) out = src0.resid[src0.row] + out;
      src0.y[src0.row] = out;
    }
  }
}

template <uint32_t TYPE, int NR>
static int launch_t(const QmvParams& p, cudaStream_t stream, int sm_count, bool pdl,
                    std::string* msg) {
  const uint32_t bb = block_bytes_of(TYPE);
  const uint32_t rb = p.cols / 256 * bb;
  const uint32_t slot_one = (rb + 32 + 127) & ~127u;
  const uint32_t slot_bytes = slot_one * NR;
  const uint32_t xbytes = 4 * (p.cols + p.cols / 16 + p.cols / 32);
  // bars (16 B per slot) + x region, rounded to 128; then slots.
  uint32_t nslots = kMaxSlots;
  uint32_t slots_off = 0, total = 0;
  for (; nslots >= 2; --nslots) {
    slots_off = (16 * nslots + xbytes + 127) & ~127u;
    total = slots_off + nslots * slot_bytes;
    if (total <= kMaxDynSmem) break;
  }
  if (nslots < 2) {
    if (msg) *msg = "matvec row is too long for the shared-memory staging ring";
    return SI_E_UNSUPPORTED;
  }
  static bool attr_set[2] = {false, false};
  (void)attr_set;
  cudaError_t e = cudaFuncSetAttribute(qmv_kernel<TYPE, NR>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMaxDynSmem));
  if (e != cudaSuccess) {
    if (msg) *msg = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
    return SI_E_CUDA;
  }
  const uint32_t grid = p.items < uint32_t(sm_count) ? p.items : uint32_t(sm_count);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, qmv_kernel<TYPE, NR>, p, slot_bytes, nslots, slots_off);
  if (e != cudaSuccess) {
    if (msg) *msg = std::string("matvec launch: ") + cudaGetErrorString(e);
    return SI_E_CUDA;
  }
  return SI_OK;
}

int launch_qmv(const QmvParams& p, cudaStream_t stream, int sm_count, bool pdl,
               std::string* msg) {
  if (p.cols == 0 || p.cols % 256 || p.cols > kQmvMaxCols || p.items == 0 || p.nseg == 0 ||
      p.nseg > 4) {
    if (msg) *msg = "matvec dimensions are invalid";
    return SI_E_INVALID;
  }
  if (p.xmode == XM_GATED && (p.head_dim == 0 || p.head_dim % 32 || p.cols % p.head_dim)) {
    if (msg) *msg = "gated-norm head dimension is invalid";
    return SI_E_INVALID;
  }
  const bool pair = p.pair != 0;
  switch (p.type) {
    case SI_GGML_TYPE_Q4_K:
      return pair ? launch_t<SI_GGML_TYPE_Q4_K, 2>(p, stream, sm_count, pdl, msg)
                  : launch_t<SI_GGML_TYPE_Q4_K, 1>(p, stream, sm_count, pdl, msg);
    case SI_GGML_TYPE_Q5_K:
      return pair ? launch_t<SI_GGML_TYPE_Q5_K, 2>(p, stream, sm_count, pdl, msg)
                  : launch_t<SI_GGML_TYPE_Q5_K, 1>(p, stream, sm_count, pdl, msg);
    case SI_GGML_TYPE_Q6_K:
      return pair ? launch_t<SI_GGML_TYPE_Q6_K, 2>(p, stream, sm_count, pdl, msg)
                  : launch_t<SI_GGML_TYPE_Q6_K, 1>(p, stream, sm_count, pdl, msg);
    default:
      if (msg) *msg = "unsupported quantized weight type";
      return SI_E_UNSUPPORTED;
  }
}

}  // namespace si
