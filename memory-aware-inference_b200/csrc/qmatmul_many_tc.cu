// Batched Q4_K / Q5_K / Q6_K matvec on the tensor cores: Y[k] = W X[k] for k < K <= 8 with
// one traversal of W (the verifier's weight pass, src/metal.rs:1055-1127,
// 4067-4230; qwen35_runtime.rs:879-1289), exact integer sub-block sums.
//
// Inputs as integers (the scheme of the batch-1 kernel, qmatvec_tc.cu): per
// candidate k and 256-column block b, X = rint(x 2^(21-e)) with e the exponent
// of the block's largest |x|, split into three signed base-256 digits
// D0 + 256 D1 + 65536 D2. A prep kernel writes them plane-major as the B
// operands of mma.m16n8k32 (u8 x s8 -> s32): MMA p of a 32-element sub-block
// takes digit plane p of candidates 0..7 as its 8 columns. The C fragment of
// each MMA then holds, in lane (g, c), rows g and g+8 of candidates 2c and
// 2c+1 - the same (row, candidate) pairs for all three planes - so the planes
// combine and scale inside the lane, as in the batch-1 kernel. The prep
// kernel also writes each candidate's block scale 2^(e-25) and its sub-block
// sums as f16 hi/lo pairs.
//
// Main kernel: one CTA per SM (the digits of a column panel live in shared
// memory, copied in by the bulk-copy engine with one mbarrier per 256-column
// block); 16 warps. A warp owns one 16-row group at a time (or one phase of
// its blocks when a group is split between warps) and streams the group's
// Q4_K super-blocks from HBM with evict-first loads, one block ahead, the
// next blocks prefetched into L2. Per sub-block: three MMAs of the raw quants
// (low nibbles as 0..15, high nibbles masked in place as 16 q) against the
// digit planes, multiplied by the 6-bit scale in integers. Per block: the
// planes are combined and scaled by d and the candidate's block scale, and the
// min term dmin * sum_j m_j xsum_kj - a 16 x 8 by 8 x 8 product - comes from
// an f16 MMA pair (the 6-bit mins are exact in f16; the sums are hi + lo f16)
// in the same fragment layout, subtracted before the block is added to the
// running sums. The epilogue adds a group's phases in shared memory in a
// fixed order. Matrices wider than a panel (33 blocks) run as column panels
// writing partial sums that a small kernel adds in panel order.
//
// Q5_K: the Q4_K path with the 5-bit quants (nibble | high bit << 4) built in
// registers instead of the masked nibbles, and the block scale 2^(e-21).
//
// Q6_K: the int8 scales cover 16 elements, so the digits are laid out per
// 16-element group and each group and plane is one m16n8k16 MMA (lane c holds
// elements 4c..4c+3 of the group); the 6-bit quants are assembled in
// registers from the low-nibble and high-bit words (loaded as 16-bit pairs:
// 210-byte super-blocks leave rows 2-byte aligned), and the -32 offset is
// the min term sum_G 32 sc_G xsum_G, one full-k f16 MMA pair.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "qmatvec.cuh"

namespace si {

namespace {

constexpr int kQtWarps = 16;
constexpr int kQtThreads = kQtWarps * 32;
constexpr uint32_t kQtSmemMax = 227 * 1024;
// Digits of one 256-column block: Q4_K [8 sub-blocks][3 planes][8 candidates]
// [32 B]; Q6_K [16 groups][3 planes][8 candidates][16 B].
constexpr uint32_t kQtDigBlock = 8 * 3 * 256;
// Sub-block sums of one block as f16 hi/lo pairs in MMA fragment order:
// Q4_K [hi/lo][8 candidates][4 lanes] (256 B used); Q6_K [hi/lo][8][4][2].
constexpr uint32_t kQtXsBlock = 512;
constexpr uint32_t kQtPrefetch = 4;             // blocks prefetched into L2 ahead of the loads

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint2 ldw_u2(const uint8_t* p, uint64_t pol) {
  uint2 v;
  asm volatile("ld.global.nc.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;" : "=r"(v.x), "=r"(v.y) : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ uint4 ldw_u4(const uint8_t* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}


__device__ __forceinline__ uint32_t ldw_u16(const uint8_t* p, uint64_t pol) {
  unsigned short v;
  asm volatile("ld.global.nc.L2::cache_hint.u16 %0, [%1], %2;" : "=h"(v) : "l"(p), "l"(pol));
  return v;
}

// Four bytes at a 2-byte aligned address (Q6_K super-blocks are 210 B).
__device__ __forceinline__ uint32_t ldw_u32_a2(const uint8_t* p, uint64_t pol) {
  return ldw_u16(p, pol) | (ldw_u16(p + 2, pol) << 16);
}

// D = A B (k = 16, u8 x s8 -> s32, zero accumulator).
__device__ __forceinline__ void mma_u8s8_k16(int* c, uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// D += A B, f16 inputs, f32 accumulate, all 16 k used.
__device__ __forceinline__ void mma_f16_k16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                            uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_u8s8(int* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// D = A B + C, f16 inputs, f32 accumulate, k = 16 with A's and B's k 8..15 zero.
__device__ __forceinline__ void mma_f16(float* d, uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%6}, {%7,%6}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(0u), "r"(b0));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, uint32_t j) { return __byte_perm(w, 0, 0x4440 | j); }

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

struct PrepArgs {
  const float* x;
  uint64_t ldx;
  uint32_t K, nblk;
  uint32_t q6;       // 1: Q6_K layouts (16-element groups), 0: Q4_K / Q5_K
  int esc_bias;      // block scale 2^(e + esc_bias): -25 for Q4_K (the 16 q trick), -21 otherwise
  uint8_t* dig;      // [nblk][kQtDigBlock]
  float* esc;        // [nblk][8]
  uint32_t* xs16;    // [nblk][kQtXsBlock / 4]
};

// One warp per (block, candidate slot 0..7); slots >= K write zeros.
__global__ void __launch_bounds__(32) qmm_prep_kernel(const PrepArgs a) {
  const uint32_t b = blockIdx.x, k = blockIdx.y, lane = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const bool live = k < a.K;
  float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (live) {
    const float4* xp = reinterpret_cast<const float4*>(a.x + k * a.ldx + b * 256 + lane * 8);
    const float4 u0 = xp[0], u1 = xp[1];
    v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
    v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
  }
  float mx = 0.f, s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mx = fmaxf(mx, fabsf(v[i]));
    s += v[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  s += __shfl_xor_sync(0xffffffffu, s, 1);  // Q6_K: group lane / 2, in both lanes of the pair
  float s16 = s;
  s += __shfl_xor_sync(0xffffffffu, s, 2);  // Q4_K: sub-block lane / 4, in every lane of the quad
  int e = int((__float_as_uint(mx) >> 23) & 255u) - 127;
  e = min(max(e, -100), 126);
  const float up = __uint_as_float(uint32_t(21 - e + 127) << 23);  // 2^(21-e), exact
  // sums in units of 2^e (|s| < 64 for a 32-element sub-block): in f16 range
  // whatever the input's magnitude; the kernels fold 2^e back in
  const float unit = __uint_as_float(uint32_t(127 - e) << 23);
  s *= unit;
  s16 *= unit;
  uint32_t pl[3][2] = {};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int X = __float2int_rn(v[i] * up);
    const int d0 = ((X + 128) & 255) - 128;
    const int X1 = (X - d0) >> 8;
    const int d1 = ((X1 + 128) & 255) - 128;
    const int d2 = (X1 - d1) >> 8;
    pl[0][i >> 2] |= uint32_t(d0 & 255) << (8 * (i & 3));
    pl[1][i >> 2] |= uint32_t(d1 & 255) << (8 * (i & 3));
    pl[2][i >> 2] |= uint32_t(d2 & 255) << (8 * (i & 3));
  }
  uint8_t* blk = a.dig + uint64_t(b) * kQtDigBlock;
  uint32_t* xs = a.xs16 + uint64_t(b) * (kQtXsBlock / 4);
  if (!a.q6) {
    const uint32_t j = lane >> 2, c = lane & 3;
#pragma unroll
    for (int p = 0; p < 3; ++p)
      *reinterpret_cast<uint2*>(blk + (j * 3 + p) * 256 + k * 32 + 8 * c) = make_uint2(pl[p][0], pl[p][1]);
    // 2^(e-21) per digit unit and 1/16 for the high nibbles being multiplied
    // as 16 q (the low-nibble scales are multiplied by 16)
    if (lane == 0) a.esc[uint64_t(b) * 8 + k] = live ? __uint_as_float(uint32_t(e + a.esc_bias + 127) << 23) : 0.f;
    // sub-block sums j = 2q, 2q+1 as f16 hi + lo pairs: the min-term MMA's B
    // fragment of lane (g = k, c = q)
    const float s_next = __shfl_down_sync(0xffffffffu, s, 4);  // sum of sub-block j + 1
    if ((lane & 7) == 0) {
      const uint32_t q = lane >> 3;
      const float h0 = __half2float(__float2half_rn(s)), h1 = __half2float(__float2half_rn(s_next));
      xs[(0 * 8 + k) * 4 + q] = pack_f16x2(h0, h1);
      xs[(1 * 8 + k) * 4 + q] = pack_f16x2(s - h0, s_next - h1);
    }
  } else {
    const uint32_t G = lane >> 1;  // 16-element group of this lane's 8 elements
#pragma unroll
    for (int p = 0; p < 3; ++p)
      *reinterpret_cast<uint2*>(blk + (G * 3 + p) * 128 + k * 16 + 8 * (lane & 1)) = make_uint2(pl[p][0], pl[p][1]);
    if (lane == 0) a.esc[uint64_t(b) * 8 + k] = live ? __uint_as_float(uint32_t(e - 21 + 127) << 23) : 0.f;
    // group sums G = 2c, 2c+1 (b0) and 2c+8, 2c+9 (b1) of the full-k f16
    // MMA's B fragment of lane (g = k, c), as hi + lo pairs
    const float s_next = __shfl_down_sync(0xffffffffu, s16, 2);  // sum of group G + 1
    if ((lane & 3) == 0) {
      const uint32_t c = (lane & 15) >> 2, slot = lane >> 4;
      const float h0 = __half2float(__float2half_rn(s16)), h1 = __half2float(__float2half_rn(s_next));
      xs[((0 * 8 + k) * 4 + c) * 2 + slot] = pack_f16x2(h0, h1);
      xs[((1 * 8 + k) * 4 + c) * 2 + slot] = pack_f16x2(s16 - h0, s_next - h1);
    }
  }
}

struct QtArgs {
  const uint8_t* w;
  const uint8_t* w_end;  // one past the matrix (the Q6_K L2 prefetch stays inside)
  uint32_t rows, nblk, K;
  const uint8_t* dig;
  const float* esc;
  const uint32_t* xs16;
  uint32_t pb;          // blocks per panel
  uint32_t nctas;       // CTAs per panel
  uint32_t ngroups;     // 16-row groups
  float* y;
  uint64_t ldy;
  const float* resid;
  uint64_t ldr;
  float* part;          // [panels][K][rows] when there is more than one panel
  uint32_t red_off;     // byte offset of the epilogue scratch in shared memory
  int* err;
};

template <uint32_t TYPE>
__global__ void __launch_bounds__(kQtThreads, 1) qmm_tc_kernel(const QtArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t panel = blockIdx.y, b0 = panel * a.pb, nb = min(a.pb, a.nblk - b0);
  uint8_t* sdig = sm;
  float* sesc = reinterpret_cast<float*>(sdig + nb * kQtDigBlock);
  uint32_t* sxs = reinterpret_cast<uint32_t*>(sesc + nb * 8);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sxs + nb * (kQtXsBlock / 4));
  float* red = reinterpret_cast<float*>(sm + a.red_off);  // [warp][16 rows][8 candidates]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;

  // groups of this CTA and their split between warps
  const uint32_t cta = blockIdx.x;
  const uint32_t g0 = uint32_t(uint64_t(cta) * a.ngroups / a.nctas);
  const uint32_t g1 = uint32_t(uint64_t(cta + 1) * a.ngroups / a.nctas);
  const uint32_t ng = g1 - g0;
  const uint32_t ngmax = (a.ngroups + a.nctas - 1) / a.nctas;
  const uint32_t split = ngmax >= kQtWarps ? 1u : min(uint32_t(kQtWarps) / ngmax, max(nb, 1u));
  const uint32_t lanes_g = kQtWarps / split;  // groups in flight per CTA

  // the digits and tables are the prep kernel's output; the residual and the
  // outputs are shared with earlier kernels: wait for all of them first
  pdl_wait();
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < nb; ++i) mbar_init(&bar[i], 1);
    fence_barrier_init();
    const uint64_t pol = l2_policy_evict_last();
    // the panel's scale tables ride on block 0's barrier, then the digits
    const uint32_t tab = nb * 32 + nb * kQtXsBlock;
    mbar_arrive_expect_tx(&bar[0], tab + kQtDigBlock);
    bulk_g2s(sesc, a.esc + uint64_t(b0) * 8, nb * 32, &bar[0], pol);
    bulk_g2s(sxs, a.xs16 + uint64_t(b0) * (kQtXsBlock / 4), nb * kQtXsBlock, &bar[0], pol);
    bulk_g2s(sdig, a.dig + uint64_t(b0) * kQtDigBlock, kQtDigBlock, &bar[0], pol);
    for (uint32_t i = 1; i < nb; ++i) {
      mbar_arrive_expect_tx(&bar[i], kQtDigBlock);
      bulk_g2s(sdig + i * kQtDigBlock, a.dig + uint64_t(b0 + i) * kQtDigBlock, kQtDigBlock, &bar[i], pol);
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  const uint64_t wpol = l2_policy_evict_first();
  const uint32_t phase = uint32_t(warp) % split;
  bool timed_out = false, table_ready = false;
  for (uint32_t gl = uint32_t(warp) / split, round = 0; round * lanes_g < ngmax; ++round, gl += lanes_g) {
    const bool active = gl < ng && !timed_out;
    // C-fragment layout: [0] row g cand 2c, [1] row g cand 2c+1, [2] row g+8
    // cand 2c, [3] row g+8 cand 2c+1
    float yk[4] = {0.f, 0.f, 0.f, 0.f};
    if (active && TYPE == SI_GGML_TYPE_Q6_K) {
      const uint32_t grp = g0 + gl;
      const uint32_t r0 = min(grp * 16 + g, a.rows - 1), r8 = min(grp * 16 + g + 8, a.rows - 1);
      const uint8_t* w0 = a.w + (uint64_t(r0) * a.nblk + b0) * 210;
      const uint8_t* w8 = a.w + (uint64_t(r8) * a.nblk + b0) * 210;
      // lanes 0..15 prefetch the 16-byte aligned envelope of row grp*16+lane's
      // blocks ahead into L2 (never past the matrix)
      const uint8_t* wp = a.w + (uint64_t(min(grp * 16 + (lane & 15), a.rows - 1)) * a.nblk + b0) * 210;
      auto prefetch = [&](uint32_t blk) {
        const uint8_t* env = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(wp + blk * 210) & ~uintptr_t(15));
        if (env + 224 <= a.w_end) prefetch_l2(env, 224);
      };
      if (lane < 16)
        for (uint32_t d = 0; d <= kQtPrefetch; ++d)
          if (phase + d * split < nb) prefetch(phase + d * split);
      for (uint32_t i = phase; i < nb; i += split) {
        if (lane < 16 && i + (kQtPrefetch + 1) * split < nb) prefetch(i + (kQtPrefetch + 1) * split);
        const uint8_t* p0 = w0 + i * 210;
        const uint8_t* p8 = w8 + i * 210;
        // int8 scales (bytes 192..207) and d (208) of rows g and g+8
        uint32_t sw0[4], sw8[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          sw0[t] = ldw_u32_a2(p0 + 192 + 4 * t, wpol);
          sw8[t] = ldw_u32_a2(p8 + 192 + 4 * t, wpol);
        }
        const float dd0 = half_bits_to_float(ldw_u16(p0 + 208, wpol));
        const float dd8 = half_bits_to_float(ldw_u16(p8 + 208, wpol));
        // quants: per half and 16-element half-group, the low-bit words of
        // m = 0,2 and m = 1,3 and the high-bit word, 4 bytes for lane c
        uint32_t ql0[2][2][2], ql8[2][2][2], qh0[2][2], qh8[2][2];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            qh0[hf][hh] = ldw_u32_a2(p0 + 128 + hf * 32 + 16 * hh + 4 * c, wpol);
            qh8[hf][hh] = ldw_u32_a2(p8 + 128 + hf * 32 + 16 * hh + 4 * c, wpol);
#pragma unroll
            for (int mp = 0; mp < 2; ++mp) {
              ql0[hf][mp][hh] = ldw_u32_a2(p0 + hf * 64 + mp * 32 + 16 * hh + 4 * c, wpol);
              ql8[hf][mp][hh] = ldw_u32_a2(p8 + hf * 64 + mp * 32 + 16 * hh + 4 * c, wpol);
            }
          }
        if (!table_ready) {
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bar[0], 0))) {
            timed_out = true;
            break;
          }
          table_ready = true;
        }
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bar[i], 0))) {
          timed_out = true;
          break;
        }
        int acc[3][4];
#pragma unroll
        for (int p = 0; p < 3; ++p) acc[p][0] = acc[p][1] = acc[p][2] = acc[p][3] = 0;
        const uint8_t* xb = sdig + i * kQtDigBlock + g * 16 + 4 * c;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
#pragma unroll
          for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int G = hf * 8 + 2 * m + hh;  // 16-element group: scale index and digit row
              const uint32_t l0 = ql0[hf][m & 1][hh], l8 = ql8[hf][m & 1][hh];
              const uint32_t a0 = (m < 2 ? (l0 & 0x0F0F0F0Fu) : ((l0 >> 4) & 0x0F0F0F0Fu)) |
                                  (((qh0[hf][hh] >> (2 * m)) & 0x03030303u) << 4);
              const uint32_t a8 = (m < 2 ? (l8 & 0x0F0F0F0Fu) : ((l8 >> 4) & 0x0F0F0F0Fu)) |
                                  (((qh8[hf][hh] >> (2 * m)) & 0x03030303u) << 4);
              const int s0 = int(int8_t(uint8_t(byte_of(sw0[G >> 2], G & 3))));
              const int s8 = int(int8_t(uint8_t(byte_of(sw8[G >> 2], G & 3))));
#pragma unroll
              for (int p = 0; p < 3; ++p) {
                const uint32_t bb = *reinterpret_cast<const uint32_t*>(xb + (G * 3 + p) * 128);
                int C[4];
                mma_u8s8_k16(C, a0, a8, bb);
                acc[p][0] += s0 * C[0];
                acc[p][1] += s0 * C[1];
                acc[p][2] += s8 * C[2];
                acc[p][3] += s8 * C[3];
              }
            }
        // the -32 offset: sum over groups of 32 sc_G (exact in f16) times the
        // group sums (f16 hi + lo), f32 accumulate
        float mt[4] = {0.f, 0.f, 0.f, 0.f};
        {
          auto sc32 = [](uint32_t w, uint32_t j) { return 32.f * float(int(int8_t(uint8_t(byte_of(w, j))))); };
          const bool hi = c >= 2;  // groups 2c, 2c+1 (word c/2) and 2c+8, 2c+9 (word 2 + c/2)
          const uint32_t jl = (2 * c) & 3;
          const uint32_t w00 = hi ? sw0[1] : sw0[0], w08 = hi ? sw8[1] : sw8[0];
          const uint32_t w20 = hi ? sw0[3] : sw0[2], w28 = hi ? sw8[3] : sw8[2];
          const uint32_t a0 = pack_f16x2(sc32(w00, jl), sc32(w00, jl + 1));
          const uint32_t a1 = pack_f16x2(sc32(w08, jl), sc32(w08, jl + 1));
          const uint32_t a2 = pack_f16x2(sc32(w20, jl), sc32(w20, jl + 1));
          const uint32_t a3 = pack_f16x2(sc32(w28, jl), sc32(w28, jl + 1));
          const uint2 bh = *reinterpret_cast<const uint2*>(sxs + i * (kQtXsBlock / 4) + ((0 * 8 + g) * 4 + c) * 2);
          const uint2 bl = *reinterpret_cast<const uint2*>(sxs + i * (kQtXsBlock / 4) + ((1 * 8 + g) * 4 + c) * 2);
          mma_f16_k16(mt, a0, a1, a2, a3, bh.x, bh.y);
          mma_f16_k16(mt, a0, a1, a2, a3, bl.x, bl.y);
        }
        const float2 es = *reinterpret_cast<const float2*>(sesc + i * 8 + 2 * c);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float f = fmaf(65536.f, float(acc[2][v]), fmaf(256.f, float(acc[1][v]), float(acc[0][v])));
          // esc = 2^(e-21) per digit unit; the sums are in units of 2^e = esc 2^21
          yk[v] += (v < 2 ? dd0 : dd8) * ((v & 1 ? es.y : es.x) * fmaf(-2097152.f, mt[v], f));
        }
      }
    }
    if (active && (TYPE == SI_GGML_TYPE_Q4_K || TYPE == SI_GGML_TYPE_Q5_K)) {
      // Q5_K: the Q4_K layout plus a high-bit plane (qh, bytes 16..47) before
      // the nibbles (bytes 48..175)
      constexpr bool q5 = TYPE == SI_GGML_TYPE_Q5_K;
      constexpr uint32_t BB = q5 ? 176 : 144, QS = q5 ? 48 : 16;
      const uint32_t grp = g0 + gl;
      const uint32_t r0 = min(grp * 16 + g, a.rows - 1), r8 = min(grp * 16 + g + 8, a.rows - 1);
      const uint8_t* w0 = a.w + (uint64_t(r0) * a.nblk + b0) * BB;
      const uint8_t* w8 = a.w + (uint64_t(r8) * a.nblk + b0) * BB;
      // lanes 0..15 prefetch row grp*16+lane of the blocks ahead into L2
      const uint8_t* wp = a.w + (uint64_t(min(grp * 16 + (lane & 15), a.rows - 1)) * a.nblk + b0) * BB;
      if (lane < 16)
        for (uint32_t d = 1; d <= kQtPrefetch + 1; ++d)
          if (phase + d * split < nb) prefetch_l2(wp + (phase + d * split) * BB, BB);
      uint4 h0, h8;
      uint2 q0[4], q8[4], qh0 = make_uint2(0u, 0u), qh8 = make_uint2(0u, 0u);
      auto load = [&](uint32_t i) {
        h0 = ldw_u4(w0 + i * BB, wpol);
        h8 = ldw_u4(w8 + i * BB, wpol);
        if (q5) {
          qh0 = ldw_u2(w0 + i * BB + 16 + 8 * c, wpol);
          qh8 = ldw_u2(w8 + i * BB + 16 + 8 * c, wpol);
        }
#pragma unroll
        for (int gr = 0; gr < 4; ++gr) {
          q0[gr] = ldw_u2(w0 + i * BB + QS + 32 * gr + 8 * c, wpol);
          q8[gr] = ldw_u2(w8 + i * BB + QS + 32 * gr + 8 * c, wpol);
        }
      };
      uint32_t i = phase;
      if (i < nb) load(i);
      for (; i < nb; i += split) {
        const uint4 ch0 = h0, ch8 = h8;
        const uint2 cqh0 = qh0, cqh8 = qh8;
        uint2 cq0[4], cq8[4];
#pragma unroll
        for (int gr = 0; gr < 4; ++gr) {
          cq0[gr] = q0[gr];
          cq8[gr] = q8[gr];
        }
        if (i + split < nb) load(i + split);  // one block ahead in registers
        if (lane < 16 && i + (kQtPrefetch + 2) * split < nb)
          prefetch_l2(wp + (i + (kQtPrefetch + 2) * split) * BB, BB);
        // the decision to stop is the warp's (its lanes then run MMAs together)
        if (!table_ready) {
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bar[0], 0))) {
            timed_out = true;
            break;
          }
          table_ready = true;
        }
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bar[i], 0))) {
          timed_out = true;
          break;
        }
        // 6-bit scales / mins of rows g and g+8 (bytes 4..15 of the header)
        uint32_t sc_lo[2], sc_hi[2], mn_lo[2], mn_hi[2];
        {
          const uint32_t w[2][3] = {{ch0.y, ch0.z, ch0.w}, {ch8.y, ch8.z, ch8.w}};
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            sc_lo[r] = w[r][0] & 0x3F3F3F3Fu;
            mn_lo[r] = w[r][1] & 0x3F3F3F3Fu;
            sc_hi[r] = (w[r][2] & 0x0F0F0F0Fu) | ((w[r][0] >> 2) & 0x30303030u);
            mn_hi[r] = ((w[r][2] >> 4) & 0x0F0F0F0Fu) | ((w[r][1] >> 2) & 0x30303030u);
          }
        }
        int acc[3][4];
#pragma unroll
        for (int p = 0; p < 3; ++p) acc[p][0] = acc[p][1] = acc[p][2] = acc[p][3] = 0;
        const uint8_t* xb = sdig + i * kQtDigBlock + g * 32 + 8 * c;
#pragma unroll
        for (int gr = 0; gr < 4; ++gr) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t j = 2 * gr + h;
            uint32_t A[4];
            int m0 = int(byte_of(j < 4 ? sc_lo[0] : sc_hi[0], j & 3));
            int m8 = int(byte_of(j < 4 ? sc_lo[1] : sc_hi[1], j & 3));
            if (q5) {
              // 5-bit quants 0..31: the nibble plus bit j of the high-bit bytes
              auto q5w = [&](uint32_t w, uint32_t hb) {
                return (h ? ((w >> 4) & 0x0F0F0F0Fu) : (w & 0x0F0F0F0Fu)) | (((hb >> j) & 0x01010101u) << 4);
              };
              A[0] = q5w(cq0[gr].x, cqh0.x);
              A[1] = q5w(cq8[gr].x, cqh8.x);
              A[2] = q5w(cq0[gr].y, cqh0.y);
              A[3] = q5w(cq8[gr].y, cqh8.y);
            } else {
              const uint32_t mask = h ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
              A[0] = cq0[gr].x & mask;
              A[1] = cq8[gr].x & mask;
              A[2] = cq0[gr].y & mask;
              A[3] = cq8[gr].y & mask;
              m0 <<= h ? 0 : 4;
              m8 <<= h ? 0 : 4;
            }
#pragma unroll
            for (int p = 0; p < 3; ++p) {
              const uint2 bb = *reinterpret_cast<const uint2*>(xb + (j * 3 + p) * 256);
              int C[4];
              mma_u8s8(C, A, bb.x, bb.y);
              acc[p][0] += m0 * C[0];
              acc[p][1] += m0 * C[1];
              acc[p][2] += m8 * C[2];
              acc[p][3] += m8 * C[3];
            }
          }
        }
        // min term: rows x sub-blocks (6-bit mins, exact in f16) times
        // sub-blocks x candidates (sums as f16 hi + lo), f32 accumulate
        float mt[4] = {0.f, 0.f, 0.f, 0.f};
        {
          const uint32_t ml0 = c < 2 ? mn_lo[0] : mn_hi[0], ml8 = c < 2 ? mn_lo[1] : mn_hi[1];
          const uint32_t jj = (2 * c) & 3;
          const uint32_t a0 = pack_f16x2(float(byte_of(ml0, jj)), float(byte_of(ml0, jj + 1)));
          const uint32_t a1 = pack_f16x2(float(byte_of(ml8, jj)), float(byte_of(ml8, jj + 1)));
          const uint32_t* xs = sxs + i * (kQtXsBlock / 4);
          mma_f16(mt, a0, a1, xs[(0 * 8 + g) * 4 + c]);
          mma_f16(mt, a0, a1, xs[(1 * 8 + g) * 4 + c]);
        }
        const float2 dd0 = __half22float2(*reinterpret_cast<const __half2*>(&ch0.x));
        const float2 dd8 = __half22float2(*reinterpret_cast<const __half2*>(&ch8.x));
        const float2 es = *reinterpret_cast<const float2*>(sesc + i * 8 + 2 * c);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float f = fmaf(65536.f, float(acc[2][v]), fmaf(256.f, float(acc[1][v]), float(acc[0][v])));
          const float d = v < 2 ? dd0.x : dd8.x, dm = v < 2 ? dd0.y : dd8.y;
          // esc = 2^(e-25) for Q4_K (digit unit / 16), 2^(e-21) for Q5_K; the
          // sums are in units of 2^e
          const float e1 = v & 1 ? es.y : es.x;
          yk[v] += d * e1 * f - dm * (e1 * (q5 ? 2097152.f : 33554432.f)) * mt[v];
        }
      }
    }
    // combine: the CTA's warps meet here once per round
    float* wr = red + warp * (16 * 8);
    if (gl < ng) {
      wr[g * 8 + 2 * c] = yk[0];
      wr[g * 8 + 2 * c + 1] = yk[1];
      wr[(g + 8) * 8 + 2 * c] = yk[2];
      wr[(g + 8) * 8 + 2 * c + 1] = yk[3];
    }
    __syncthreads();
    // outputs of this round: lanes_g groups x 16 rows x K candidates
    for (uint32_t o = threadIdx.x; o < lanes_g * 16 * a.K; o += kQtThreads) {
      const uint32_t k = o % a.K, row = (o / a.K) % 16, slot = o / (16 * a.K);
      const uint32_t glo = slot + round * lanes_g;
      if (glo >= ng) continue;
      const uint32_t r = (g0 + glo) * 16 + row;
      if (r >= a.rows) continue;
      float v = 0.f;
      for (uint32_t ph = 0; ph < split; ++ph) v += red[(slot * split + ph) * (16 * 8) + row * 8 + k];
      if (gridDim.y > 1) {
        a.part[(uint64_t(panel) * a.K + k) * a.rows + r] = v;
      } else {
        const float base = a.resid ? a.resid[k * a.ldr + r] : 0.f;
        a.y[k * a.ldy + r] = base + v;
      }
    }
    __syncthreads();
  }
  // no copy may still be landing when the CTA retires (bounded)
  if (threadIdx.x == 0)
    for (uint32_t bi = 0; bi < nb; ++bi)
      if (!mbar_wait_bounded(&bar[bi], 0)) {
        if (a.err) atomicOr(a.err, KERR_TIMEOUT_DRAIN);
        break;
      }
  if (timed_out && a.err) atomicOr(a.err, KERR_TIMEOUT_FULL);
}

// Panel sums in panel order, then the residual.
__global__ void qmm_reduce_kernel(const float* part, uint32_t panels, uint32_t K, uint32_t rows, float* y,
                                  uint64_t ldy, const float* resid, uint64_t ldr) {
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x, k = blockIdx.y;
  if (r >= rows) return;
  float v = 0.f;
  for (uint32_t p = 0; p < panels; ++p) v += part[(uint64_t(p) * K + k) * rows + r];
  y[k * ldy + r] = (resid ? resid[k * ldr + r] : 0.f) + v;
}

struct Geometry {
  uint32_t pb, panels, nctas, smem, red_off;
  uint64_t dig_bytes, esc_bytes, xs_bytes, part_bytes;
};

Geometry geometry(uint32_t rows, uint32_t cols, uint32_t K, int sm_count) {
  Geometry g = {};
  const uint32_t nblk = cols / 256;
  const uint32_t per_blk = kQtDigBlock + 32 + kQtXsBlock + 8;
  const uint32_t red = kQtWarps * 16 * 8 * 4;
  const uint32_t pb = std::max(1u, (kQtSmemMax - red - 256) / per_blk);
  g.panels = (nblk + pb - 1) / pb;
  g.pb = (nblk + g.panels - 1) / g.panels;  // balanced panels
  const uint32_t groups = (rows + 15) / 16;
  g.nctas = std::max(1u, std::min(groups, uint32_t(std::max(1, sm_count)) / g.panels));
  g.red_off = (g.pb * per_blk + 64 + 127) & ~127u;
  g.smem = g.red_off + red;
  g.dig_bytes = uint64_t(nblk) * kQtDigBlock;
  g.esc_bytes = uint64_t(nblk) * 32;
  g.xs_bytes = uint64_t(nblk) * kQtXsBlock;
  g.part_bytes = g.panels > 1 ? uint64_t(g.panels) * K * rows * 4 : 0;
  return g;
}

uint64_t align256u(uint64_t v) { return (v + 255) & ~uint64_t(255); }

}  // namespace

uint64_t qmm_tc_scratch_bytes(uint32_t rows, uint32_t cols, uint32_t batch, int sm_count) {
  const Geometry g = geometry(rows, cols, batch, sm_count);
  return align256u(g.dig_bytes) + align256u(g.esc_bytes) + align256u(g.xs_bytes) + align256u(g.part_bytes);
}

bool qmm_tc_eligible(const QmmParams& p) {
  const bool q6 = p.type == SI_GGML_TYPE_Q6_K;
  const bool k4 = p.type == SI_GGML_TYPE_Q4_K || p.type == SI_GGML_TYPE_Q5_K;  // 16-byte loads
  return (k4 || q6) && p.batch >= 2 && p.batch <= kQmmMaxBatch && p.rows >= 16 &&
         !(reinterpret_cast<uintptr_t>(p.w) & (k4 ? 15u : 1u)) && p.scratch &&
         !(reinterpret_cast<uintptr_t>(p.scratch) & 255);
}

int launch_qmm_tc(const QmmParams& p, cudaStream_t s, int sm_count, bool pdl, std::string* msg) {
  const Geometry g = geometry(p.rows, p.cols, p.batch, sm_count);
  if (qmm_tc_scratch_bytes(p.rows, p.cols, p.batch, sm_count) > p.scratch_bytes) return SI_E_UNSUPPORTED;
  uint8_t* sc = static_cast<uint8_t*>(p.scratch);
  PrepArgs pa = {};
  pa.x = p.x;
  pa.ldx = p.ldx;
  pa.K = p.batch;
  pa.nblk = p.cols / 256;
  pa.q6 = p.type == SI_GGML_TYPE_Q6_K;
  pa.esc_bias = p.type == SI_GGML_TYPE_Q4_K ? -25 : -21;
  pa.dig = sc;
  pa.esc = reinterpret_cast<float*>(sc + align256u(g.dig_bytes));
  pa.xs16 = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(pa.esc) + align256u(g.esc_bytes));
  float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(pa.xs16) + align256u(g.xs_bytes));

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pa.nblk, 8);  // every candidate slot: unused ones write zeros
  cfg.blockDim = dim3(32);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qmm_prep_kernel, pa);

  QtArgs a = {};
  a.w = p.w;
  a.w_end = p.w + uint64_t(p.rows) * pa.nblk * block_bytes_of(p.type);
  a.rows = p.rows;
  a.nblk = pa.nblk;
  a.K = p.batch;
  a.dig = pa.dig;
  a.esc = pa.esc;
  a.xs16 = pa.xs16;
  a.pb = g.pb;
  a.nctas = g.nctas;
  a.ngroups = (p.rows + 15) / 16;
  a.y = p.y;
  a.ldy = p.ldy;
  a.resid = p.resid;
  a.ldr = p.ldr;
  a.part = part;
  a.red_off = g.red_off;
  a.err = p.err;
  const int ti = p.type == SI_GGML_TYPE_Q4_K ? 0 : p.type == SI_GGML_TYPE_Q5_K ? 1 : 2;
  auto kern = ti == 0 ? qmm_tc_kernel<SI_GGML_TYPE_Q4_K>
            : ti == 1 ? qmm_tc_kernel<SI_GGML_TYPE_Q5_K>
                      : qmm_tc_kernel<SI_GGML_TYPE_Q6_K>;
  if (e == cudaSuccess) {
    static std::atomic<uint32_t> smem_limit[3][kMaxDevices];  // per type and device
    e = raise_smem_limit(kern, kQtSmemMax, smem_limit[ti]);
  }
  if (e == cudaSuccess) {
    cudaLaunchConfig_t mc = {};
    mc.gridDim = dim3(g.nctas, g.panels);
    mc.blockDim = dim3(kQtThreads);
    mc.dynamicSmemBytes = g.smem;
    mc.stream = s;
    mc.attrs = attr;
    mc.numAttrs = 1;  // after the prep kernel: its tail overlaps this prologue
    e = cudaLaunchKernelEx(&mc, kern, a);
  }
  if (e == cudaSuccess && g.panels > 1) {
    qmm_reduce_kernel<<<dim3((p.rows + 255) / 256, p.batch), 256, 0, s>>>(part, g.panels, p.batch, p.rows, p.y,
                                                                           p.ldy, p.resid, p.ldr);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    if (msg) *msg = std::string("batched tensor-core matvec launch: ") + cudaGetErrorString(e);
    return SI_E_CUDA;
  }
  return SI_OK;
}

}  // namespace si
