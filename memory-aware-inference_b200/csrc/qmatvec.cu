// Batch-1 GGUF K-quant matvec for sm_100a.
//
// Replaces the Metal kernels si_q4_k_matvec / si_q5_k_matvec / si_q6_k_matvec
// (+ their rows4 variants), si_q4_k_fused_gate_up and the grouped matvec
// (src/metal.rs:310-494, 498-587, 770-1050, 4532-4780 in the reference).
//
// Design (two CTAs per SM, each persistent over a contiguous range of rows):
//  * Each CTA has 7 consumer warps and 1 producer warp. Lane t of the
//    producer warp issues team t's copies: rows (a whole 2,880 B Q4_K
//    5120-column row, or an adjacent pair of rows, merged into one copy)
//    stream from HBM into shared-memory slots with non-tensor bulk async
//    copies (cp.async.bulk, L2 evict_first), tracked by full/empty
//    mbarriers. Each team owns >= 2 private slots (double buffering), so
//    barrier phases never alias.
//  * A team is 16 (or 32) lanes and owns NR = 2 rows that share every load of
//    x. Lane l of a team always decodes the same 64-element unit of each
//    super-block (Q4_K/Q5_K: group l%4; Q6_K: half/16-run l%4), so the 6-bit
//    scale/min extraction pattern is fixed per lane and never diverges.
//  * Q4_K: x is converted once per launch, in shared memory, into exact
//    24-bit fixed-point byte planes per 32-element sub-block (scale 2^(e-22)
//    for the sub-block's largest exponent e); each sub-block dot product is
//    an exact integer sum of dp4a instructions on the raw nibbles, scaled back
//    in fp32 and accumulated across sub-blocks in fp32.
//  * Q5_K / Q6_K: each quant q is placed in the low mantissa byte of 2^23
//    (PRMT, no int->float conversion pipe), 2^23 is subtracted exactly in
//    pairs (fadd.rn.f32x2), and q*x is accumulated by packed fp32 FMA
//    (fma.rn.f32x2).
//  * The min / -32 offsets are applied per sub-block with precomputed
//    sub-block sums of x. The input vector x (and an optional fused RMSNorm /
//    gated-norm / sigmoid-gate transform of it) lives in shared memory.
//    Epilogues: store, residual add, SwiGLU pair.
//  * Team results are combined with transposed warp-shuffle reductions.
//    Tensor cores are not used: batch-1 is not a contraction.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "qmatvec.cuh"

namespace si {

// Two CTAs per SM, each 7 consumer warps + 1 producer: 16 warps per SM (4 per
// scheduler, up to 128 registers per thread). While one CTA of a kernel
// drains, a CTA of the next kernel in the stream (programmatic dependent
// launch) already initialises and prefetches its weights in the other half.
constexpr int kCtasPerSm = 2;
constexpr int kConsumerWarps = 7;
constexpr int kThreads = kConsumerWarps * 32 + 32;
constexpr int kMaxTeams = kConsumerWarps * 2;
constexpr int kTeamLanes = 16;
constexpr int kMaxSlots = 64;
constexpr uint32_t kPieceBytes = 4608;  // target bytes of one staged row piece
constexpr float kBias = 8388608.0f;     // 2^23

// Per-format constants. x lives in shared memory with 4 floats of padding
// after every 2^kPad elements, which makes the float4 loads of the 8 lanes
// of a quarter-warp hit 8 disjoint bank groups for each format's lane map.
template <uint32_t TYPE>
struct Fmt;
template <>
struct Fmt<SI_GGML_TYPE_Q4_K> {
  static constexpr uint32_t BB = 144, kPad = 6, kSum = 32;
};
template <>
struct Fmt<SI_GGML_TYPE_Q5_K> {
  static constexpr uint32_t BB = 176, kPad = 6, kSum = 32;
};
template <>
struct Fmt<SI_GGML_TYPE_Q6_K> {
  static constexpr uint32_t BB = 210, kPad = 7, kSum = 16;
};

template <uint32_t PAD>
__device__ __forceinline__ uint32_t xi(uint32_t e) {
  return e + 4u * (e >> PAD);
}

// Byte j of `word` as the float 2^23 + byte (exact); subtracting 2^23 (in
// pairs, fadd.rn.f32x2) leaves the integer exactly.
__device__ __forceinline__ float bias_float(uint32_t word, int j) {
  return as_f(__byte_perm(word, 0x4B000000u, 0x7440u | uint32_t(j)));
}

__device__ __forceinline__ float2 int_pair(uint32_t word, int j) {
  return __fadd2_rn(make_float2(bias_float(word, j), bias_float(word, j + 1)),
                    make_float2(-kBias, -kBias));
}

__device__ __forceinline__ float small_uint_to_float(uint32_t v) {
  return as_f(0x4B000000u | v) - kBias;  // v < 2^23, exact, no conversion pipe
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// 16 bytes from a 2-byte-aligned shared-memory address.
__device__ __forceinline__ uint4 lds16_a2(const uint8_t* p) {
  const uint32_t off = smem_u32(p) & 3u;
  const uint32_t* w = reinterpret_cast<const uint32_t*>(p - off);
  const uint32_t a = w[0], b = w[1], c = w[2], d = w[3], e = w[4];
  const uint32_t sh = off * 8u;
  return make_uint4(__funnelshift_r(a, b, sh), __funnelshift_r(b, c, sh),
                    __funnelshift_r(c, d, sh), __funnelshift_r(d, e, sh));
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// 6-bit scale/min pairs (2g, 2g+1) of a K-quant header (quant.rs:176-185),
// with lane-constant g, as floats.
struct ScalePairs {
  float sa, sb, ma, mb;
};

__device__ __forceinline__ ScalePairs k4_scales(const uint4& hdr, int g) {
  // Branch-free (g is lane-constant but differs within a warp).
  const uint32_t W1 = hdr.y, W2 = hdr.z, W3 = hdr.w;
  const bool lowg = g < 2;
  const uint32_t sh = 16u * uint32_t(g & 1);
  const uint32_t A = lowg ? W1 : W3, B = lowg ? W2 : (W3 >> 4);
  const uint32_t m6 = lowg ? 63u : 15u, hm = lowg ? 0u : 0x30u;
  const uint32_t sa = ((A >> sh) & m6) | ((W1 >> (sh + 2)) & hm);
  const uint32_t sb = ((A >> (sh + 8)) & m6) | ((W1 >> (sh + 10)) & hm);
  const uint32_t ma = ((B >> sh) & m6) | ((W2 >> (sh + 2)) & hm);
  const uint32_t mb = ((B >> (sh + 8)) & m6) | ((W2 >> (sh + 10)) & hm);
  const float2 s2 = __fadd2_rn(make_float2(as_f(0x4B000000u | sa), as_f(0x4B000000u | sb)),
                               make_float2(-kBias, -kBias));
  const float2 m2 = __fadd2_rn(make_float2(as_f(0x4B000000u | ma), as_f(0x4B000000u | mb)),
                               make_float2(-kBias, -kBias));
  ScalePairs s;
  s.sa = s2.x;
  s.sb = s2.y;
  s.ma = m2.x;
  s.mb = m2.y;
  return s;
}

// ---------------------------------------------------------------------------
// Unit decoders. A unit is 64 weights of one super-block that a lane owns:
// Q4_K/Q5_K group g = lane%4 (quant bytes 32g..32g+31: low nibbles are
// elements 64g+0..31, high nibbles 64g+32..63); Q6_K half h and 16-run i0
// with (h, i0/16) = lane%4. Each computes sum_i w_i x_i for NR rows that
// share x.
// ---------------------------------------------------------------------------
template <uint32_t TYPE>
struct Unit;

__device__ __forceinline__ uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Q4_K with integer sub-block dot products. x is held per 32-element
// sub-block j as X_i = rint(x_i * 2^(22-e_j)) (|X| < 2^22, the block's
// largest element keeps a full 23-bit significand) split into three byte
// planes (two unsigned, the top one signed); sum_i q_i X_i is computed exactly
// with dp4a (int32, no overflow: 32 * 240 * 255 < 2^31) and scaled back by
// 2^(e_j-22) in fp32. The quants of one x load serve NR rows.
template <>
struct Unit<SI_GGML_TYPE_Q4_K> {
  // NU independent units (blocks bb[0..NU)) of NR rows each; one x load
  // serves the NR rows. blk[v * NR + r] is unit v of row r.
  template <int NR, int NU = 1>
  __device__ __forceinline__ static void run(const uint8_t* const* blk, const float* xs,
                                             const float* xsum, const uint32_t* bb, int l4,
                                             float* acc, uint32_t nsub) {
    const int g = l4;
    uint4 hdr[NU][NR], qa[NU][NR], qb[NU][NR];
#pragma unroll
    for (int v = 0; v < NU; ++v)
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        hdr[v][r] = lds128(blk[v * NR + r]);
        qa[v][r] = lds128(blk[v * NR + r] + 16 + 32 * g);
        qb[v][r] = lds128(blk[v * NR + r] + 32 + 32 * g);
      }
    uint32_t l0[NU][NR], l1[NU][NR], h0[NU][NR], h1[NU][NR];
    int l2[NU][NR], h2[NU][NR];
#pragma unroll
    for (int v = 0; v < NU; ++v)
#pragma unroll
      for (int r = 0; r < NR; ++r) l0[v][r] = l1[v][r] = h0[v][r] = h1[v][r] = 0u, l2[v][r] = h2[v][r] = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
#pragma unroll
      for (int v = 0; v < NU; ++v) {
        const uint4* xq = reinterpret_cast<const uint4*>(xs) + (68 * bb[v] + 17 * g);
        const uint4 xl = xq[k], xh = xq[8 + k];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
          const uint32_t w = word_of(k < 4 ? qa[v][r] : qb[v][r], k & 3);
          const uint32_t lo = w & 0x0F0F0F0Fu;  // q
          const uint32_t hi = w & 0xF0F0F0F0u;  // 16 q
          l0[v][r] = dp4a_uu(lo, xl.x, l0[v][r]);
          l1[v][r] = dp4a_uu(lo, xl.y, l1[v][r]);
          l2[v][r] = dp4a_us(lo, xl.z, l2[v][r]);
          h0[v][r] = dp4a_uu(hi, xh.x, h0[v][r]);
          h1[v][r] = dp4a_uu(hi, xh.y, h1[v][r]);
          h2[v][r] = dp4a_us(hi, xh.z, h2[v][r]);
        }
      }
    }
#pragma unroll
    for (int v = 0; v < NU; ++v) {
      const uint32_t b = bb[v];
      const float Xl = xsum[b * 8 + g * 2], Xh = xsum[b * 8 + g * 2 + 1];
      const float* sc = xsum + nsub;
      const float sl = sc[b * 8 + g * 2], shs = sc[b * 8 + g * 2 + 1] * 0.0625f;
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        const float Sl = (float(l2[v][r]) * 65536.0f + float(int(l1[v][r] * 256u + l0[v][r]))) * sl;
        const float Sh = (float(h2[v][r]) * 65536.0f + float(int(h1[v][r] * 256u + h0[v][r]))) * shs;
        const ScalePairs s = k4_scales(hdr[v][r], g);
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hdr[v][r].x));
        acc[r] += dm.x * (s.sa * Sl + s.sb * Sh) - dm.y * (s.ma * Xl + s.mb * Xh);
      }
    }
  }
};

template <>
struct Unit<SI_GGML_TYPE_Q5_K> {
  template <int NR, int NU = 1>
  __device__ __forceinline__ static void run(const uint8_t* const* blk, const float* xs,
                                             const float* xsum, const uint32_t* bb, int l4,
                                             float* acc, uint32_t /*nsub*/) {
    const uint32_t b = bb[0];
    const int g = l4;
    const float* xp = xs + xi<6>(b * 256 + g * 64);
    const float Xl = xsum[b * 8 + g * 2], Xh = xsum[b * 8 + g * 2 + 1];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const uint4 hdr = lds128(blk[r]);
      const uint4 ha = lds128(blk[r] + 16), hb = lds128(blk[r] + 32);
      const uint4 qa = lds128(blk[r] + 48 + 32 * g), qb = lds128(blk[r] + 64 + 32 * g);
      float2 l0 = make_float2(0.f, 0.f), l1 = l0, h0 = l0, h1 = l0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 xl = *reinterpret_cast<const float4*>(xp + 4 * k);
        const float4 xh = *reinterpret_cast<const float4*>(xp + 32 + 4 * k);
        const uint32_t w = word_of(k < 4 ? qa : qb, k & 3);
        const uint32_t h = word_of(k < 4 ? ha : hb, k & 3);
        const uint32_t lo = (w & 0x0F0F0F0Fu) | (((h >> (2 * g)) & 0x01010101u) << 4);
        const uint32_t hi = ((w >> 4) & 0x0F0F0F0Fu) | (((h >> (2 * g + 1)) & 0x01010101u) << 4);
        l0 = __ffma2_rn(int_pair(lo, 0), make_float2(xl.x, xl.y), l0);
        l1 = __ffma2_rn(int_pair(lo, 2), make_float2(xl.z, xl.w), l1);
        h0 = __ffma2_rn(int_pair(hi, 0), make_float2(xh.x, xh.y), h0);
        h1 = __ffma2_rn(int_pair(hi, 2), make_float2(xh.z, xh.w), h1);
      }
      const float Sl = (l0.x + l0.y) + (l1.x + l1.y);
      const float Sh = (h0.x + h0.y) + (h1.x + h1.y);
      const ScalePairs s = k4_scales(hdr, g);
      const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hdr.x));
      acc[r] += dm.x * (s.sa * Sl + s.sb * Sh) - dm.y * (s.ma * Xl + s.mb * Xh);
    }
  }
};

template <>
struct Unit<SI_GGML_TYPE_Q6_K> {
  template <int NR, int NU = 1>
  __device__ __forceinline__ static void run(const uint8_t* const* blk, const float* xs,
                                             const float* xsum, const uint32_t* bb, int l4,
                                             float* acc, uint32_t /*nsub*/) {
    const uint32_t b = bb[0];
    const int h = l4 >> 1, i0 = (l4 & 1) * 16;
    const uint32_t e0 = b * 256 + 128 * h + i0;
    const float* xp = xs + xi<7>(e0);
    float X[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) X[m] = xsum[(e0 >> 4) + 2 * m];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const uint8_t* bp = blk[r];
      const uint4 L1 = lds16_a2(bp + 64 * h + i0);
      const uint4 L2 = lds16_a2(bp + 64 * h + 32 + i0);
      const uint4 H = lds16_a2(bp + 128 + 32 * h + i0);
      const uint8_t* scp = bp + 192 + 8 * h + (l4 & 1);
      const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(bp + 208));
      float2 a[4], c[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) a[m] = c[m] = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t l1 = word_of(L1, k), l2 = word_of(L2, k), hh = word_of(H, k);
        uint32_t v[4];
        v[0] = (l1 & 0x0F0F0F0Fu) | ((hh << 4) & 0x30303030u);
        v[1] = (l2 & 0x0F0F0F0Fu) | ((hh << 2) & 0x30303030u);
        v[2] = ((l1 >> 4) & 0x0F0F0F0Fu) | (hh & 0x30303030u);
        v[3] = ((l2 >> 4) & 0x0F0F0F0Fu) | ((hh >> 2) & 0x30303030u);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float4 xv = *reinterpret_cast<const float4*>(xp + 32 * m + 4 * k);
          a[m] = __ffma2_rn(int_pair(v[m], 0), make_float2(xv.x, xv.y), a[m]);
          c[m] = __ffma2_rn(int_pair(v[m], 2), make_float2(xv.z, xv.w), c[m]);
        }
      }
      float t = 0.f;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float sc = float(int(static_cast<int8_t>(scp[2 * m])));
        const float S = (a[m].x + a[m].y) + (c[m].x + c[m].y);  // sum q x, q in 0..63
        t += sc * (S - 32.0f * X[m]);
      }
      acc[r] += d * t;
    }
  }
};

// ---------------------------------------------------------------------------
// Launch geometry (computed on the host).
// ---------------------------------------------------------------------------
struct QmvGeom {
  uint32_t mode;          // 0 single row, 1 SwiGLU pair, 2 two independent rows
  uint32_t merge;         // adjacent row pairs may be staged by one copy
  uint32_t team_lanes;    // 16 or 32 lanes per team
  uint32_t items;         // work items (mode 2: row pairs)
  uint32_t piece_blocks;  // super-blocks per staged piece (multiple of 4)
  uint32_t npieces;       // pieces per row
  uint32_t slot_bytes;    // bytes of one slot (NR rows)
  uint32_t row_slot;      // bytes reserved per row inside a slot
  uint32_t nslots, teams, per_team;
  uint32_t slots_off;     // shared-memory offset of the slots
  uint32_t xs_floats;     // padded x length
};

struct SegSm {
  const uint8_t* w;
  float* y;
  const float* resid;
  uint32_t rows;
};

// Row `which` (0..NR-1) of work item `item`: pair mode = gate/up row `item`;
// dual mode = rows 2*item and 2*item+1 (the odd tail repeats its row and
// skips the second store); single mode = row `item`. Segments (grouped
// matvec) are looked up in the shared-memory table.
struct RowRef {
  const uint8_t* g;
  float* y;
  const float* resid;
  uint32_t row;
  bool store;
};

__device__ __forceinline__ RowRef row_ref(const SegSm* seg, uint32_t nseg, uint32_t mode,
                                          uint32_t total, uint32_t item, uint32_t rb, int which,
                                          uint32_t nr) {
  RowRef r;
  r.store = true;
  if (mode == 1) {  // SwiGLU pair
    r.g = seg[which].w + size_t(item) * rb;
    r.y = seg[0].y;
    r.resid = seg[0].resid;
    r.row = item;
    return r;
  }
  uint32_t v = item;
  if (mode == 2) {
    v = nr * item + uint32_t(which);
    if (v >= total) {
      v = total - 1;
      r.store = false;
    }
  }
  if (nseg == 1) {
    r.g = seg[0].w + size_t(v) * rb;
    r.y = seg[0].y;
    r.resid = seg[0].resid;
    r.row = v;
    return r;
  }
  uint32_t k = 0;
  while (k + 1 < nseg && v >= seg[k].rows) {
    v -= seg[k].rows;
    ++k;
  }
  r.g = seg[k].w + size_t(v) * rb;
  r.y = seg[k].y;
  r.resid = seg[k].resid;
  r.row = v;
  return r;
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// Team t of a CTA owns slots [t*per_team, (t+1)*per_team) and processes rows
// t, t+teams, ... of the CTA's range, each as npieces pieces; its j-th piece
// uses slot t*per_team + j % per_team in round j / per_team. Only the owning
// team waits on a slot's full barrier, strictly in round order, so a waiter
// is never more than one phase ahead of the barrier.
template <uint32_t TYPE, int NR>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    qmv_kernel(const __grid_constant__ QmvParams p, const __grid_constant__ QmvGeom G) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_abort;
  __shared__ float s_red[kConsumerWarps];
  __shared__ SegSm s_seg[4];
  constexpr uint32_t BB = Fmt<TYPE>::BB;
  constexpr uint32_t PAD = Fmt<TYPE>::kPad;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + G.nslots;
  const uint32_t cols = p.cols;
  float* xs = reinterpret_cast<float*>(smem + 16 * G.nslots);
  float* xsum = xs + G.xs_floats;
  uint8_t* slots = smem + G.slots_off;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t nb = cols / 256;
  const uint32_t rb = nb * BB;
  const uint32_t i0 = uint32_t(uint64_t(blockIdx.x) * G.items / gridDim.x);
  const uint32_t i1 = uint32_t(uint64_t(blockIdx.x + 1) * G.items / gridDim.x);
  const uint32_t n_items = i1 - i0;
  const uint32_t T = G.teams, M = G.per_team, NP = G.npieces, P = G.piece_blocks;
  const uint32_t nseg = p.nseg, mode = G.mode, total = p.items;

  for (uint32_t s = threadIdx.x; s < G.nslots; s += blockDim.x) {
    mbar_init(&full[s], 1);
    mbar_init(&empty[s], 1);
  }
  if (threadIdx.x < 4) {
    const uint32_t k = threadIdx.x;
    s_seg[k].w = p.seg[k].w;
    s_seg[k].y = p.seg[k].y;
    s_seg[k].resid = p.seg[k].resid;
    s_seg[k].rows = p.seg[k].rows;
  }
  if (threadIdx.x == 0) s_abort = 0;
  if (threadIdx.x < G.nslots) fence_barrier_init();
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kConsumerWarps) {
    // ---------------- producer warp: lane t streams team t's row pieces -----
    // Each lane issues its own team's copies, so up to 32 bulk copies leave
    // per warp instruction and no team waits behind another team's slot.
    const uint32_t t = uint32_t(lane);
    if (t < T && t < n_items) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t issued = 0, pc = 0, rl = t, si = 0, round = 0;
      uintptr_t prow[NR];
      bool abort = false;
      while (rl < n_items) {
        const uint32_t s = t * M + si;
        if (round > 0 && !mbar_wait_bounded(&empty[s], (round - 1) & 1)) {
          atomicOr(p.err, KERR_TIMEOUT_EMPTY);
          s_abort = 1;
          abort = true;
          break;
        }
        if (*reinterpret_cast<volatile int*>(&s_abort)) {
          abort = true;
          break;
        }
        const uint32_t b0 = pc * P, pb = min(P, nb - b0);
        uintptr_t a0[NR], a1[NR];
        static_assert(NR <= 4, "four rows per slot at most");
        uint32_t tx = 0;
#pragma unroll
        for (int w = 0; w < NR; ++w) {
          if (pc == 0) prow[w] = reinterpret_cast<uintptr_t>(row_ref(s_seg, nseg, mode, total, i0 + rl, rb, w, NR).g);
          const uintptr_t a = prow[w] + uintptr_t(b0) * BB;
          a0[w] = a & ~uintptr_t(15);
          a1[w] = (a + uintptr_t(pb) * BB + 15) & ~uintptr_t(15);
          tx += uint32_t(a1[w] - a0[w]);
        }
        uint8_t* dst = slots + size_t(s) * G.slot_bytes;
        bool adjacent = NR > 1 && G.merge;
#pragma unroll
        for (int w = 0; w + 1 < NR; ++w) adjacent = adjacent && (a1[w] == a0[w + 1]);
        if (adjacent) {
          // adjacent rows land as one copy (row w at dst + w * row_slot, row_slot = rb)
          mbar_arrive_expect_tx(&full[s], uint32_t(a1[NR - 1] - a0[0]));
          bulk_g2s(dst, reinterpret_cast<const void*>(a0[0]), uint32_t(a1[NR - 1] - a0[0]), &full[s], pol);
        } else {
          mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
          for (int w = 0; w < NR; ++w)
            bulk_g2s(dst + w * G.row_slot, reinterpret_cast<const void*>(a0[w]), uint32_t(a1[w] - a0[w]),
                     &full[s], pol);
        }
        ++issued;
        if (++pc == NP) {
          pc = 0;
          rl += T;
        }
        if (++si == M) {
          si = 0;
          ++round;
        }
      }
      if (abort) {
        // Drain: wait (bounded) for this team's copies still in flight.
        for (uint32_t q = 0; q < M && q < issued; ++q) {
          const uint32_t j = issued - 1 - q;
          if (!mbar_wait_bounded(&full[t * M + j % M], (j / M) & 1)) atomicOr(p.err, KERR_TIMEOUT_DRAIN);
        }
      }
    }
    return;
  }

  // ---------------- consumers: build x (padded layout) in shared memory ----
  pdl_wait();
  const int ct = threadIdx.x;
  constexpr int NC = kConsumerWarps * 32;
  if (p.xmode == XM_RAW || p.xmode == XM_RMS1P) {
    // all loads of a chunk are issued before any store (latency overlap)
    float ss = 0.f;
    for (uint32_t base = ct * 4; base < cols; base += NC * 4 * 4) {
      float4 v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t i = base + q * NC * 4;
        v[q] = i < cols ? *reinterpret_cast<const float4*>(p.x + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t i = base + q * NC * 4;
        if (i < cols) {
          *reinterpret_cast<float4*>(xs + xi<PAD>(i)) = v[q];
          ss += v[q].x * v[q].x + v[q].y * v[q].y + v[q].z * v[q].z + v[q].w * v[q].w;
        }
      }
    }
    if (p.xmode == XM_RMS1P) {
      ss = warp_sum(ss);
      if (lane == 0) s_red[warp] = ss;
      consumer_sync();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) tot += s_red[w];
      const float inv = 1.0f / sqrtf(tot / float(cols) + p.eps);
      for (uint32_t i = ct; i < cols; i += NC) {
        const uint32_t k = xi<PAD>(i);
        xs[k] = xs[k] * inv * (1.0f + p.xw[i]);
      }
    }
  } else if (p.xmode == XM_GATED) {
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
        xs[xi<PAD>(h * hd + i)] = v * inv * p.xw[i] * (z / (1.0f + expf(-z)));
      }
    }
  } else {  // XM_SIGGATE
    for (uint32_t i = ct; i < cols; i += NC) {
      const float gte = p.xaux[i];
      xs[xi<PAD>(i)] = p.x[i] / (1.0f + expf(-gte));
    }
  }
  consumer_sync();
  constexpr uint32_t SUM = Fmt<TYPE>::kSum;
  for (uint32_t j = ct; j < cols / SUM; j += NC) {
    float* q = xs + xi<PAD>(SUM * j);
    float4 v[SUM / 4];
    float t = 0.f, m = 0.f;
#pragma unroll
    for (uint32_t i = 0; i < SUM / 4; ++i) {
      v[i] = *reinterpret_cast<const float4*>(q + 4 * i);
      t += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
    xsum[j] = t;
    if (TYPE == SI_GGML_TYPE_Q4_K) {
      // x as 24-bit fixed point per 32-element sub-block: X = rint(x * 2^(22-e))
      // with m < 2^e, |X| <= 2^22, X = b2 * 65536 + b1 * 256 + b0; each group of
      // 4 floats is overwritten in place by {b0 x4, b1 x4, b2 x4 (signed), 0}.
      // e is clamped to [-100, 129] so 2^(22-e) and 2^(e-22) are normal floats
      // (a smaller e only lowers the resolution floor below 2^-122).
      int ex = int((__float_as_uint(m) >> 23) & 0xffu) - 126;
      ex = ex < -100 ? -100 : (ex > 129 ? 129 : ex);
      xsum[cols / 32 + j] = __uint_as_float(uint32_t(ex + 105) << 23);
      const float mul = __uint_as_float(uint32_t(149 - ex) << 23);
#pragma unroll
      for (uint32_t i = 0; i < SUM / 4; ++i) {
        const uint32_t X0 = uint32_t(__float2int_rn(v[i].x * mul)), X1 = uint32_t(__float2int_rn(v[i].y * mul));
        const uint32_t X2 = uint32_t(__float2int_rn(v[i].z * mul)), X3 = uint32_t(__float2int_rn(v[i].w * mul));
        uint4 o;
        o.x = __byte_perm(__byte_perm(X0, X1, 0x0040u), __byte_perm(X2, X3, 0x0040u), 0x5410u);
        o.y = __byte_perm(__byte_perm(X0, X1, 0x0051u), __byte_perm(X2, X3, 0x0051u), 0x5410u);
        o.z = __byte_perm(__byte_perm(X0, X1, 0x0062u), __byte_perm(X2, X3, 0x0062u), 0x5410u);
        o.w = 0u;
        *reinterpret_cast<uint4*>(q + 4 * i) = o;
      }
    }
  }
  consumer_sync();

  // ---------------- consumers: pieces of rows, per-team private slots ------
  const uint32_t TL = G.team_lanes;
  const uint32_t team = uint32_t(ct) / TL;
  const int tl = int(uint32_t(ct) % TL);
  if (team >= T) return;
  const unsigned tmask = TL == 32 ? 0xffffffffu : ((lane < 16) ? 0x0000ffffu : 0xffff0000u);
  float acc[NR];
#pragma unroll
  for (int w = 0; w < NR; ++w) acc[w] = 0.f;
  uint32_t pc = 0, rl = team, si = 0, round = 0;
  RowRef rows_g[NR];
#pragma unroll
  for (int w = 0; w < NR; ++w) rows_g[w] = RowRef{nullptr, nullptr, nullptr, 0u, false};
  while (rl < n_items) {
    const uint32_t s = team * M + si;
    if (!mbar_wait_bounded(&full[s], round & 1)) {
      atomicOr(p.err, KERR_TIMEOUT_FULL);
      s_abort = 1;
      break;
    }
    const uint32_t b0 = pc * P, pb = min(P, nb - b0);
    const uint8_t* base = slots + size_t(s) * G.slot_bytes;
    if (pc == 0) {
#pragma unroll
      for (int w = 0; w < NR; ++w) rows_g[w] = row_ref(s_seg, nseg, mode, total, i0 + rl, rb, w, NR);
    }
    const uint8_t* rowp[NR];
#pragma unroll
    for (int w = 0; w < NR; ++w)
      rowp[w] = base + w * G.row_slot + ((reinterpret_cast<uintptr_t>(rows_g[w].g) + uintptr_t(b0) * BB) & 15);
    const uint32_t units = pb * 4;
    uint32_t u = tl;
    if (TYPE == SI_GGML_TYPE_Q4_K && NR <= 2) {
      for (; u + TL < units; u += 2 * TL) {
        const uint8_t* blk[2 * NR];
        const uint32_t bb[2] = {b0 + (u >> 2), b0 + ((u + TL) >> 2)};
#pragma unroll
        for (int w = 0; w < NR; ++w) {
          blk[w] = rowp[w] + (u >> 2) * BB;
          blk[NR + w] = rowp[w] + ((u + TL) >> 2) * BB;
        }
        Unit<TYPE>::template run<NR, 2>(blk, xs, xsum, bb, tl & 3, acc, cols / 32);
      }
    }
    for (; u < units; u += TL) {
      const uint8_t* blk[NR];
#pragma unroll
      for (int w = 0; w < NR; ++w) blk[w] = rowp[w] + (u >> 2) * BB;
      const uint32_t bb[1] = {b0 + (u >> 2)};
      Unit<TYPE>::template run<NR, 1>(blk, xs, xsum, bb, tl & 3, acc, cols / 32);
    }
    __syncwarp(tmask);
    if (tl == 0) mbar_arrive(&empty[s]);
    if (++pc == NP) {
      if (NR == 2) {
        // transposed reduction: one exchange leaves row (lane & 1) in every
        // lane, then a single butterfly over the remaining lanes
        const bool odd = lane & 1;
        const float send = odd ? acc[0] : acc[NR - 1];
        const float keep = odd ? acc[NR - 1] : acc[0];
        float v = keep + __shfl_xor_sync(tmask, send, 1);
        if (TL == 32) v += __shfl_xor_sync(0xffffffffu, v, 16);
        v += __shfl_xor_sync(tmask, v, 8);
        v += __shfl_xor_sync(tmask, v, 4);
        v += __shfl_xor_sync(tmask, v, 2);
        const float other = __shfl_xor_sync(tmask, v, 1);
        acc[0] = odd ? other : v;
        acc[NR - 1] = odd ? v : other;
      } else if (NR == 4) {
        // transposed reduction of four rows: after two exchanges lane l holds
        // row (l & 3); the butterfly then sums over the remaining lanes
        const bool b0s = lane & 1, b1s = lane & 2;
        const float a = (b0s ? acc[1] : acc[0]) + __shfl_xor_sync(tmask, b0s ? acc[0] : acc[1], 1);
        const float c = (b0s ? acc[NR - 1] : acc[2]) + __shfl_xor_sync(tmask, b0s ? acc[2] : acc[NR - 1], 1);
        float v = (b1s ? c : a) + __shfl_xor_sync(tmask, b1s ? a : c, 2);
        if (TL == 32) v += __shfl_xor_sync(0xffffffffu, v, 16);
        v += __shfl_xor_sync(tmask, v, 8);
        v += __shfl_xor_sync(tmask, v, 4);
        acc[0] = v;  // row (tl & 3)
      } else {
        if (TL == 32) acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) acc[0] += __shfl_xor_sync(tmask, acc[0], o);
      }
      if (NR == 4) {
        if (tl < 4) {
#pragma unroll
          for (int w = 0; w < NR; ++w)
            if (tl == w) {
              const RowRef& rr = rows_g[w];
              if (rr.store) rr.y[rr.row] = rr.resid ? rr.resid[rr.row] + acc[0] : acc[0];
            }
        }
      } else if (tl == 0) {
        if (mode == 1) {
          const RowRef& rr = rows_g[0];
          const float gv = acc[0];
          float out = gv / (1.0f + expf(-gv)) * acc[NR - 1];
          if (rr.resid) out = rr.resid[rr.row] + out;
          rr.y[rr.row] = out;
        } else {
#pragma unroll
          for (int w = 0; w < NR; ++w) {
            const RowRef& rr = rows_g[w];
            if (rr.store) rr.y[rr.row] = rr.resid ? rr.resid[rr.row] + acc[w] : acc[w];
          }
        }
      }
#pragma unroll
      for (int w = 0; w < NR; ++w) acc[w] = 0.f;
      pc = 0;
      rl += T;
    }
    if (++si == M) {
      si = 0;
      ++round;
    }
  }
}

template <uint32_t TYPE, int NR>
static int launch_t(const QmvParams& p, cudaStream_t stream, int sm_count, bool pdl,
                    std::string* msg) {
  constexpr uint32_t BB = Fmt<TYPE>::BB;
  constexpr uint32_t PAD = Fmt<TYPE>::kPad;
  const uint32_t nb = p.cols / 256;
  QmvGeom G = {};
  // piece: a multiple of 4 super-blocks of at most ~kPieceBytes
  uint32_t P = (kPieceBytes / BB) & ~3u;
  if (P < 4) P = 4;
  if (nb <= P) P = nb;
  G.piece_blocks = P;
  G.mode = p.pair ? 1u : (NR >= 2 ? 2u : 0u);
  G.items = G.mode == 2 ? (p.items + NR - 1) / NR : p.items;
  G.npieces = (nb + P - 1) / P;
  G.row_slot = (P * BB + 32 + 127) & ~127u;
  // whole 16-byte-aligned rows in one piece: a row pair can be one copy
  if (NR >= 2 && G.npieces == 1 && (nb * BB) % 16 == 0 && G.mode == 2) {
    G.merge = 1;
    G.row_slot = nb * BB;
  }
  G.slot_bytes = G.row_slot * NR;
  G.xs_floats = p.cols + 4 * (p.cols >> PAD);
  const uint32_t xbytes = 4 * (G.xs_floats + p.cols / Fmt<TYPE>::kSum +
                                (TYPE == SI_GGML_TYPE_Q4_K ? p.cols / 32 : 0));
  // per instantiation and device: the attribute belongs to the current device
  static std::atomic<uint32_t> max_dyn_dev[kMaxDevices];
  int cur_dev = 0;
  cudaGetDevice(&cur_dev);
  std::atomic<uint32_t>& max_dyn_slot = max_dyn_dev[cur_dev >= 0 && cur_dev < kMaxDevices ? cur_dev : 0];
  uint32_t max_dyn = max_dyn_slot.load(std::memory_order_relaxed);
  if (max_dyn == 0) {
    int dev = cur_dev, optin = 0, per_sm = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    optin = std::min(optin, per_sm / kCtasPerSm - 1024);
    cudaFuncAttributes fa = {};
    cudaFuncGetAttributes(&fa, qmv_kernel<TYPE, NR>);
    const uint32_t limit = uint32_t(optin) > uint32_t(fa.sharedSizeBytes) + 256
                               ? uint32_t(optin) - uint32_t(fa.sharedSizeBytes) - 256
                               : 0;
    cudaError_t e = cudaFuncSetAttribute(qmv_kernel<TYPE, NR>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(limit));
    if (e != cudaSuccess) {
      if (msg) *msg = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
      return SI_E_CUDA;
    }
    max_dyn = limit;
    max_dyn_slot.store(limit, std::memory_order_relaxed);
  }
  // largest slot count that fits, then teams with >= 2 private slots each
  uint32_t nslots = kMaxSlots, total = 0;
  for (; nslots >= 2; --nslots) {
    G.slots_off = (16 * nslots + xbytes + 127) & ~127u;
    total = G.slots_off + nslots * G.slot_bytes;
    if (total <= max_dyn) break;
  }
  if (nslots < 2) {
    if (msg) *msg = "matvec input vector is too long for the shared-memory staging ring";
    return SI_E_UNSUPPORTED;
  }
  G.teams = nslots / 2 < uint32_t(kMaxTeams) ? nslots / 2 : uint32_t(kMaxTeams);
  G.team_lanes = kTeamLanes;
  if (G.teams <= uint32_t(kConsumerWarps) + 2) {  // one warp per team
    G.team_lanes = 32;
    G.teams = G.teams < uint32_t(kConsumerWarps) ? G.teams : uint32_t(kConsumerWarps);
  }
  G.per_team = nslots / G.teams;
  G.nslots = G.teams * G.per_team;
  G.slots_off = (16 * G.nslots + xbytes + 127) & ~127u;
  total = G.slots_off + G.nslots * G.slot_bytes;
  const uint32_t cap = uint32_t(sm_count) * kCtasPerSm;
  const uint32_t grid = G.items < cap ? G.items : cap;
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, qmv_kernel<TYPE, NR>, p, G);
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
  if (p.peer.n) {
    // the exchange lives in the tensor-core kernels, which their callers launch directly
    if (msg) *msg = "a matvec with a peer exchange goes to launch_qmv_tc or launch_qmv_tc6";
    return SI_E_UNSUPPORTED;
  }
  const bool pair = p.pair != 0;
  switch (p.type) {
    case SI_GGML_TYPE_Q4_K:
      if (!pair && p.xmode == XM_RAW && p.nseg > 1) {
        // grouped plain matvec: segment by segment, so every segment's rows are
        // exactly those of a single call on it
        for (uint32_t i = 0; i < p.nseg; ++i) {
          QmvParams q = p;
          q.nseg = 1;
          q.seg[0] = p.seg[i];
          q.items = p.seg[i].rows;
          if (int rc = launch_qmv(q, stream, sm_count, pdl, msg)) return rc;
        }
        return SI_OK;
      }
      if (qmv_tc_eligible(p)) {
        const int rc = launch_qmv_tc(p, stream, sm_count, pdl, msg);
        if (rc != SI_E_UNSUPPORTED) return rc;
      }
      // two rows per team step share each x load (SwiGLU: gate and up rows)
      return launch_t<SI_GGML_TYPE_Q4_K, 2>(p, stream, sm_count, pdl, msg);
    case SI_GGML_TYPE_Q5_K:
      return pair ? launch_t<SI_GGML_TYPE_Q5_K, 2>(p, stream, sm_count, pdl, msg)
                  : launch_t<SI_GGML_TYPE_Q5_K, 1>(p, stream, sm_count, pdl, msg);
    case SI_GGML_TYPE_Q6_K:
      if (qmv_tc6_eligible(p)) {
        const int rc = launch_qmv_tc6(p, stream, sm_count, pdl, msg);
        if (rc != SI_E_UNSUPPORTED) return rc;
      }
      return pair ? launch_t<SI_GGML_TYPE_Q6_K, 2>(p, stream, sm_count, pdl, msg)
                  : launch_t<SI_GGML_TYPE_Q6_K, 1>(p, stream, sm_count, pdl, msg);
    default:
      if (msg) *msg = "unsupported quantized weight type";
      return SI_E_UNSUPPORTED;
  }
}

}  // namespace si
