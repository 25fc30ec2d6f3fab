// Q4_K matvec y = W x on the tensor cores with exact integer sub-block sums.
//
// Same contract as qmv_kernel for a plain Q4_K matvec (src/metal.rs:310-494,
// 3357-3397, 3923 in the reference): fp32 result of sum_i w_i x_i with
// w_i = d*sc*q - dmin*m (quant.rs:18-65).
//
// x as integers. Per 256-column block b, x is scaled by 2^(21-e_b) (e_b =
// exponent of the block's largest |x|) and rounded: X_i = rint(x_i 2^(21-e_b)),
// |X_i| <= 2^22, so |x_i - X_i 2^(e_b-21)| <= 2^-22 max|x| in the block. X is
// split into three signed base-256 digits, X = D0 + 256 D1 + 65536 D2
// (D0, D1 in [-128, 127], D2 in [-64, 64]), stored in shared memory as the
// columns 0..2 of the MMA's B operand for every 32-element sub-block.
//
// Dot products. For 16 rows and one 32-element sub-block, mma.m16n8k32
// (u8 x s8 -> s32) multiplies the raw quants (low nibbles as 0..15, high
// nibbles masked in place as 16*q) by the digit columns: C[row][p] =
// sum_k q[row][k] D_p[k], exact. The 6-bit sub-block scales are applied in
// integers (acc_p += sc_j * C_p, |acc| < 2^29), the three digit columns are
// combined in fp32 once per block, and the block's d, dmin and min term
// (dmin * sum_j m_j * sum_{i in j} x_i) are applied in fp32.
//
// Data movement. Two CTAs per SM (one when the x digits of very wide rows do
// not fit twice); each CTA owns a band of 16-row groups; the consumer
// warps are shared out evenly over the groups ("split" warps per group, each
// taking every split-th 256-column block) and add their partial sums at the
// end in a fixed order. A producer lane issues one 3-D TMA per 256-column block for
// the whole band (tensor map {144 B, blocks, rows}, box {144, 1, band rows}),
// so each row of the staged tile is one 144-byte super-block: the 144-byte
// row pitch (16 mod 128) makes the fragment loads of 8 rows bank-conflict
// free. Stages are recycled through full/empty mbarriers with bounded waits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "qmatvec.cuh"
#include "peer_exchange.cuh"

namespace si {

constexpr int kTcGroups = 8;                     // 16-row groups per CTA at most
constexpr int kTcCtasPerSm = 2;
// Consumer warps; a CTA with ngmax groups gives each group kTcConsumers/ngmax
// warps ("split"), warp part p taking the blocks i = p (mod split).
constexpr int kTcConsumers = 12;
// Every warp phase owns kTcSlots private stages (double buffering): a warp
// only ever waits on a stage whose previous phase it consumed itself, so an
// mbarrier parity can never be mistaken for one a full phase ahead. A stage
// holds one 256-column block of the CTA's band (2,304 B per 16-row group), so
// the ring is kTcConsumers * kTcSlots * 2,304 B whatever the split.
constexpr int kTcSlots = 2;
constexpr uint32_t kTcGroupBlockBytes = 144 * 16;
constexpr uint32_t kTcRingBytes = kTcConsumers * kTcSlots * kTcGroupBlockBytes;
constexpr int kTcMaxStages = kTcConsumers * kTcSlots;
constexpr int kTcThreads = (kTcConsumers + 1) * 32;

constexpr uint32_t kTcMaxBlocks = 80;            // x digits: 1 KiB per block

struct TcArgs {
  const float* x;
  float* y;
  const float* resid;    // optional residual added in the epilogue (may alias y)
  const float* xw;       // XM_RMS1P: [cols] (1+w) norm weight; XM_GATED: [head_dim]
  const float* xaux;     // XM_GATED: z; XM_SIGGATE: gate
  float eps;
  int xmode;
  uint32_t head_dim;     // XM_GATED (64, 128 or 256)
  uint32_t rows, nblk, ngroups, nctas;
  uint32_t mats;         // 1, or 2 for a SwiGLU pair (gate = map 0, up = map 1)
  // two segments sharing x in one launch (mats 1, no peer output): CTAs
  // [0, nctas0) run segment 0 (maps 0, y, resid, rows, ngroups), the others
  // segment 1 (maps 1, y1, resid1, rows1, ngroups1); nctas0 = 0: one segment
  uint32_t nctas0, rows1, ngroups1;
  float* y1;
  const float* resid1;
  int* err;
  PeerOut peer;          // n > 0: the rows go to every rank's vector (NVLink stores)
};

// C = A B with a zero accumulator (no register moves to clear C).
__device__ __forceinline__ void mma_u8s8_zero(int* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void tma_load_3d_u8(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                               uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, uint32_t j) { return __byte_perm(w, 0, 0x4440 | j); }

__global__ void __launch_bounds__(kTcThreads, kTcCtasPerSm)
    qmv_tc_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                  const __grid_constant__ CUtensorMap up_hi, const __grid_constant__ CUtensorMap up_lo,
                  const __grid_constant__ TcArgs a) {
  extern __shared__ __align__(128) uint8_t tsm[];
  uint8_t* ring = tsm;                                          // stages x tile_bytes
  uint8_t* xd = ring + kTcRingBytes;                            // [blk][8 sb][4 planes][32] s8
  float* xsum = reinterpret_cast<float*>(xd + a.nblk * 1024);   // [blk][8]
  float* escale = xsum + a.nblk * 8;                            // [blk]
  uint64_t* full = reinterpret_cast<uint64_t*>(escale + ((a.nblk + 1) & ~1u));
  uint64_t* empty = full + kTcMaxStages;
  uint64_t* xready = empty + kTcMaxStages;                      // [blk]: digits of block written

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this CTA's segment, its index among the segment's CTAs, their count
  const bool seg1 = a.nctas0 != 0 && blockIdx.x >= a.nctas0;
  const uint32_t cta = seg1 ? blockIdx.x - a.nctas0 : blockIdx.x;
  const uint32_t sctas = seg1 ? a.nctas - a.nctas0 : (a.nctas0 ? a.nctas0 : a.nctas);
  const uint32_t sgroups = seg1 ? a.ngroups1 : a.ngroups;
  const uint32_t g0 = uint32_t(uint64_t(cta) * sgroups / sctas);
  const uint32_t g1 = uint32_t(uint64_t(cta + 1) * sgroups / sctas);
  const uint32_t ng = g1 - g0;                                   // 16-row groups of this CTA
  const uint32_t ngmax = (sgroups + sctas - 1) / sctas;
  const CUtensorMap* map = seg1 ? (ng == ngmax ? &up_hi : &up_lo) : (ng == ngmax ? &map_hi : &map_lo);
  const CUtensorMap* map_up = ng == ngmax ? &up_hi : &up_lo;
  float* const out_y = seg1 ? a.y1 : a.y;
  const float* const out_resid = seg1 ? a.resid1 : a.resid;
  const uint32_t out_rows = seg1 ? a.rows1 : a.rows;
  // "virtual groups": the CTA's row groups of each matrix (a SwiGLU pair has
  // the same rows of gate and up, staged one after the other)
  const uint32_t nv = ng * a.mats, nvmax = ngmax * a.mats;
  const uint32_t tile_bytes = kTcGroupBlockBytes * ng;          // one matrix
  const uint32_t split = kTcConsumers / nvmax;                  // warps per virtual group
  const uint32_t stage_bytes = kTcGroupBlockBytes * nvmax;
  // block i -> phase h = i % split, its n-th block (n = i / split) uses stage
  // h * kTcSlots + n % kTcSlots with parity (n / kTcSlots) & 1

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < split * kTcSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], nv);  // the warps of one phase consume a stage
    }
    for (uint32_t b = 0; b < a.nblk; ++b) mbar_init(&xready[b], 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kTcConsumers) {
    // ---- producer: one TMA per 256-column block for the whole band ----
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t window = split * kTcSlots;  // blocks in flight at most
      for (uint32_t i = 0; i < a.nblk; ++i) {
        const uint32_t n = i / split, s = (i % split) * kTcSlots + n % kTcSlots;
        if (n >= uint32_t(kTcSlots) && !mbar_wait_bounded(&empty[s], ((n / kTcSlots) - 1) & 1)) {
          if (a.err) atomicOr(a.err, KERR_TIMEOUT_EMPTY);
          // drain what is in flight, then stop issuing
          for (uint32_t j = (i > window ? i - window : 0); j < i; ++j) {
            const uint32_t nj = j / split, sj = (j % split) * kTcSlots + nj % kTcSlots;
            if (!mbar_wait_bounded(&full[sj], (nj / kTcSlots) & 1) && a.err) atomicOr(a.err, KERR_TIMEOUT_DRAIN);
          }
          break;
        }
        mbar_arrive_expect_tx(&full[s], tile_bytes * a.mats);
        tma_load_3d_u8(smem_u32(ring + s * stage_bytes), map, 0, int(i), int(g0 * 16), &full[s], pol);
        if (a.mats == 2)
          tma_load_3d_u8(smem_u32(ring + s * stage_bytes + tile_bytes), map_up, 0, int(i), int(g0 * 16), &full[s],
                         pol);
      }
    }
    return;
  }

  // ---- x (transformed as xmode says) -> digit planes, sub-block sums,
  //      block scales (consumer warps) ----
  pdl_wait();
  // the launch's epoch (PeerOut): the previous grid has finished, so its
  // last CTA's advance is visible
  __shared__ uint32_t s_epoch;
  if (a.peer.n && threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(a.peer.epoch) + 1;
  float rms_inv = 1.f;
  if (a.xmode == XM_RMS1P) {
    // (1+w) RMSNorm over the whole vector (qwen35.rs:53-86, heads = 1)
    __shared__ float s_red[kTcConsumers];
    float ss = 0.f;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    for (uint32_t i = threadIdx.x; i < a.nblk * 64; i += kTcConsumers * 32) {
      const float4 u = x4[i];
      ss += u.x * u.x + u.y * u.y + u.z * u.z + u.w * u.w;
    }
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    asm volatile("bar.sync 1, %0;" ::"r"(kTcConsumers * 32) : "memory");
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kTcConsumers; ++w) tot += s_red[w];
    rms_inv = 1.0f / sqrtf(tot / float(a.nblk * 256) + a.eps);
  }
  // the x loads of the warp's first two blocks leave together (one L2 round
  // trip instead of two for rows of up to 24 blocks)
  float4 pre[2][2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint32_t b = warp + k * kTcConsumers;
    if (b < a.nblk) {
      const float4* xp = reinterpret_cast<const float4*>(a.x + b * 256 + lane * 8);
      pre[k][0] = xp[0];
      pre[k][1] = xp[1];
    }
  }
  for (uint32_t b = warp, k = 0; b < a.nblk; b += kTcConsumers, ++k) {
    float v[8];
    const uint32_t e0 = b * 256 + lane * 8;
    float4 u0, u1;
    if (k == 0) {
      u0 = pre[0][0];
      u1 = pre[0][1];
    } else if (k == 1) {
      u0 = pre[1][0];
      u1 = pre[1][1];
    } else {
      const float4* xp = reinterpret_cast<const float4*>(a.x + e0);
      u0 = xp[0];
      u1 = xp[1];
    }
    v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
    v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
    if (a.xmode == XM_RMS1P) {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = v[k] * rms_inv * (1.0f + a.xw[e0 + k]);
    } else if (a.xmode == XM_GATED) {
      // per head of head_dim: x * rsqrt(mean x^2 + eps) * w[d] * SiLU(z) (qwen35.rs:14-49)
      const uint32_t hl = a.head_dim / 8;  // lanes per head (8, 16 or 32)
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += v[k] * v[k];
      for (uint32_t o = 1; o < hl; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = 1.0f / sqrtf(ss / float(a.head_dim) + a.eps);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float z = a.xaux[e0 + k];
        v[k] = v[k] * inv * a.xw[(e0 + k) % a.head_dim] * (z / (1.0f + expf(-z)));
      }
    } else if (a.xmode == XM_SIGGATE) {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = v[k] / (1.0f + expf(-a.xaux[e0 + k]));
    }
    float mx = 0.f, s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      mx = fmaxf(mx, fabsf(v[k]));
      s += v[k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    int e = int((__float_as_uint(mx) >> 23) & 255u) - 127;   // exponent of the block max
    e = max(e, -100);
    const float up = __uint_as_float(uint32_t(21 - e + 127) << 23);    // 2^(21-e), exact
    uint32_t pl[3][2] = {};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int X = __float2int_rn(v[k] * up);
      const int d0 = ((X + 128) & 255) - 128;
      const int X1 = (X - d0) >> 8;
      const int d1 = ((X1 + 128) & 255) - 128;
      const int d2 = (X1 - d1) >> 8;
      pl[0][k >> 2] |= uint32_t(d0 & 255) << (8 * (k & 3));
      pl[1][k >> 2] |= uint32_t(d1 & 255) << (8 * (k & 3));
      pl[2][k >> 2] |= uint32_t(d2 & 255) << (8 * (k & 3));
    }
    // plane p of sub-block sb sits at slot (p + sb) % 4 of the sub-block's
    // 128 bytes: the fragment loads stay contiguous, the stores spread banks
    const uint32_t sb = lane >> 2, k0 = (lane & 3) * 8;
    uint8_t* dst = xd + (b * 8 + sb) * 128 + k0;
#pragma unroll
    for (int p = 0; p < 3; ++p)
      *reinterpret_cast<uint2*>(dst + ((p + sb) & 3) * 32) = make_uint2(pl[p][0], pl[p][1]);
    *reinterpret_cast<uint2*>(dst + ((3 + sb) & 3) * 32) = make_uint2(0u, 0u);
    if ((lane & 3) == 0) xsum[b * 8 + sb] = s;
    // 2^(e-21) / 16: high-nibble sub-blocks are multiplied as 16 q
    if (lane == 0) escale[b] = __uint_as_float(uint32_t(e - 21 - 4 + 127) << 23);
    __syncwarp();
    if (lane == 0) mbar_arrive(&xready[b]);  // release: this block's digits, sums and scale
  }

  const int g = lane >> 2, c = lane & 3;
  float yg = 0.f, yg8 = 0.f;
  const uint32_t vgrp = uint32_t(warp) / split, half = uint32_t(warp) % split;  // half: block phase
  const bool active = vgrp < nv;
  const uint32_t mat = active ? vgrp / ng : 0, grp_w = active ? vgrp % ng : vgrp;
  // row of this lane inside a stage: matrix `mat`'s tile, then its group
  const uint32_t row_in_band = mat * ng * 16 + grp_w * 16 + g;
  // lane offset of digit plane g inside a sub-block, for sub-block index j mod 4
  uint32_t boff[4];
#pragma unroll
  for (int jm = 0; jm < 4; ++jm) boff[jm] = ((g + jm) & 3) * 32 + 8 * c;
  for (uint32_t i = half, n = 0; i < a.nblk; i += split, ++n) {  // n: this phase's block count
    const uint32_t s = half * kTcSlots + n % kTcSlots;
    if (!active) break;
    if (!mbar_wait_bounded(&full[s], (n / kTcSlots) & 1)) {
      if (a.err) atomicOr(a.err, KERR_TIMEOUT_FULL);
      break;
    }
    if (!mbar_wait_bounded(&xready[i], 0)) {
      if (a.err) atomicOr(a.err, KERR_TIMEOUT_FULL);
      break;
    }
    const uint8_t* r0 = ring + s * stage_bytes + row_in_band * 144;
    const uint8_t* r8 = r0 + 8 * 144;
    // header: d, dmin (f16 pair), 12 bytes of packed 6-bit scales / mins
    const uint32_t h0 = *reinterpret_cast<const uint32_t*>(r0), h8 = *reinterpret_cast<const uint32_t*>(r8);
    uint32_t sc_lo[2], sc_hi[2], mn_lo[2], mn_hi[2];
    {
      const uint32_t* p0 = reinterpret_cast<const uint32_t*>(r0 + 4);
      const uint32_t* p8 = reinterpret_cast<const uint32_t*>(r8 + 4);
      const uint32_t w[2][3] = {{p0[0], p0[1], p0[2]}, {p8[0], p8[1], p8[2]}};
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        sc_lo[r] = w[r][0] & 0x3F3F3F3Fu;
        mn_lo[r] = w[r][1] & 0x3F3F3F3Fu;
        sc_hi[r] = (w[r][2] & 0x0F0F0F0Fu) | ((w[r][0] >> 2) & 0x30303030u);
        mn_hi[r] = ((w[r][2] >> 4) & 0x0F0F0F0Fu) | ((w[r][1] >> 2) & 0x30303030u);
      }
    }
    int acc[4] = {0, 0, 0, 0};
    const uint8_t* xb = xd + i * 1024;
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      // k <-> element map: lane c's k = 4c..4c+3 are elements 8c..8c+3 and its
      // k = 16+4c..16+4c+3 are elements 8c+4..8c+7, for A and B alike, so both
      // operands are one 8-byte load per lane (the sum over k is unchanged)
      const uint32_t off = 16 + 32 * grp + 8 * c;
      const uint2 q0 = *reinterpret_cast<const uint2*>(r0 + off);
      const uint2 q8 = *reinterpret_cast<const uint2*>(r8 + off);
      const uint32_t qa0 = q0.x, qb0 = q0.y, qa8 = q8.x, qb8 = q8.y;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t j = 2 * grp + h;  // sub-block
        const uint32_t mask = h ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
        const uint32_t A[4] = {qa0 & mask, qa8 & mask, qb0 & mask, qb8 & mask};
        uint32_t b0 = 0, b1 = 0;
        if (g < 4) {
          const uint2 bb = *reinterpret_cast<const uint2*>(xb + j * 128 + boff[j & 3]);
          b0 = bb.x;
          b1 = bb.y;
        }
        int C[4];
        mma_u8s8_zero(C, A, b0, b1);
        const int m0 = int(byte_of(j < 4 ? sc_lo[0] : sc_hi[0], j & 3)) << (h ? 0 : 4);
        const int m8 = int(byte_of(j < 4 ? sc_lo[1] : sc_hi[1], j & 3)) << (h ? 0 : 4);
        acc[0] += m0 * C[0];
        acc[1] += m0 * C[1];
        acc[2] += m8 * C[2];
        acc[3] += m8 * C[3];
      }
    }
    // digit columns: lane c=0 holds D0, D1; lane c=1 holds D2 (and a zero column)
    float f0 = c == 0 ? fmaf(256.f, float(acc[1]), float(acc[0])) : (c == 1 ? 65536.f * float(acc[0]) : 0.f);
    float f8 = c == 0 ? fmaf(256.f, float(acc[3]), float(acc[2])) : (c == 1 ? 65536.f * float(acc[2]) : 0.f);
    f0 += __shfl_xor_sync(0xffffffffu, f0, 1);
    f8 += __shfl_xor_sync(0xffffffffu, f8, 1);
    // min term: lane c takes sub-blocks 2c, 2c+1 of both rows, then the quad sums
    const float* xs = xsum + i * 8 + 2 * c;
    const uint32_t ml0 = c < 2 ? mn_lo[0] : mn_hi[0], ml8 = c < 2 ? mn_lo[1] : mn_hi[1];
    const uint32_t jj = (2 * c) & 3;
    float mt0 = float(byte_of(ml0, jj)) * xs[0] + float(byte_of(ml0, jj + 1)) * xs[1];
    float mt8 = float(byte_of(ml8, jj)) * xs[0] + float(byte_of(ml8, jj + 1)) * xs[1];
    mt0 += __shfl_xor_sync(0xffffffffu, mt0, 1);
    mt8 += __shfl_xor_sync(0xffffffffu, mt8, 1);
    mt0 += __shfl_xor_sync(0xffffffffu, mt0, 2);
    mt8 += __shfl_xor_sync(0xffffffffu, mt8, 2);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (c == 0) {
      const float es = escale[i];
      const float2 dd0 = __half22float2(*reinterpret_cast<const __half2*>(&h0));
      const float2 dd8 = __half22float2(*reinterpret_cast<const __half2*>(&h8));
      yg += dd0.x * es * f0 - dd0.y * mt0;
      yg8 += dd8.x * es * f8 - dd8.y * mt8;
    }
  }
  // the other phases hand their sums to the phase-0 warp of their group
  float* red = reinterpret_cast<float*>(ring);  // every stage has been consumed
  float* upv = red + kTcConsumers * kTcGroups * 16;  // SwiGLU: up-row totals
  static_assert((kTcConsumers + 1) * kTcGroups * 16 * 4 <= kTcRingBytes, "reduction buffer");
  asm volatile("bar.sync 1, %0;" ::"r"(kTcConsumers * 32) : "memory");
  if (half > 0 && active && c == 0) {
    red[((half - 1) * kTcGroups + vgrp) * 16 + g] = yg;
    red[((half - 1) * kTcGroups + vgrp) * 16 + g + 8] = yg8;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kTcConsumers * 32) : "memory");
  if (half == 0 && active && c == 0) {
    for (uint32_t h = 1; h < split; ++h) {
      yg += red[((h - 1) * kTcGroups + vgrp) * 16 + g];
      yg8 += red[((h - 1) * kTcGroups + vgrp) * 16 + g + 8];
    }
    if (mat == 1) {
      upv[grp_w * 16 + g] = yg;
      upv[grp_w * 16 + g + 8] = yg8;
    }
  }
  if (a.mats == 2) asm volatile("bar.sync 1, %0;" ::"r"(kTcConsumers * 32) : "memory");
  if (half == 0 && active && c == 0 && mat == 0) {
    const uint32_t row = (g0 + grp_w) * 16 + g;
    float o0 = yg, o8 = yg8;
    if (a.mats == 2) {  // SwiGLU: SiLU(gate) * up (metal.rs:498-587)
      o0 = yg / (1.0f + expf(-yg)) * upv[grp_w * 16 + g];
      o8 = yg8 / (1.0f + expf(-yg8)) * upv[grp_w * 16 + g + 8];
    }
    if (a.peer.n) {
      if (row < out_rows) peer_store_row(a.peer, s_epoch, row, out_resid ? out_resid[row] + o0 : o0);
      if (row + 8 < out_rows) peer_store_row(a.peer, s_epoch, row + 8, out_resid ? out_resid[row + 8] + o8 : o8);
    } else {
      if (row < out_rows) out_y[row] = out_resid ? out_resid[row] + o0 : o0;
      if (row + 8 < out_rows) out_y[row + 8] = out_resid ? out_resid[row + 8] + o8 : o8;
    }
  }
  if (a.peer.n) peer_gather(a.peer, a.nctas, s_epoch, a.err, kTcConsumers * 32);
}

static PFN_cuTensorMapEncodeTiled_v12000 tc_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Tensor map over Q4_K rows viewed as [rows][blocks][144 B], box {144, 1, band}.
static bool q4k_band_map(CUtensorMap* m, const void* w, uint32_t rows, uint32_t nblk, uint32_t band) {
  auto enc = tc_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(w) & 15) || band == 0 || band > 256) return false;
  const cuuint64_t dims[3] = {144, nblk, rows};
  const cuuint64_t strides[2] = {144, cuuint64_t(nblk) * 144};
  const cuuint32_t box[3] = {144, 1, band};
  const cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(w), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Q4_K matvecs with any x transform, residual epilogue and SwiGLU pairing; a
// grouped call becomes one launch per segment (pairs: one launch), so every
// row matches a single call on its segment bit for bit.
bool qmv_tc_supported(const QmvParams& p) {
  if (p.type != SI_GGML_TYPE_Q4_K || p.cols / 256 > kTcMaxBlocks || (reinterpret_cast<uintptr_t>(p.x) & 15))
    return false;
  if (p.xmode == XM_GATED && p.head_dim != 64 && p.head_dim != 128 && p.head_dim != 256) return false;
  if ((p.xmode == XM_RMS1P || p.xmode == XM_GATED) && !p.xw) return false;
  if ((p.xmode == XM_GATED || p.xmode == XM_SIGGATE) && !p.xaux) return false;
  if (p.pair && (p.nseg != 2 || p.seg[0].rows != p.seg[1].rows)) return false;
  for (uint32_t i = 0; i < p.nseg; ++i)
    if ((reinterpret_cast<uintptr_t>(p.seg[i].w) & 15) || p.seg[i].rows < 16) return false;
  return true;
}

bool qmv_tc_eligible(const QmvParams& p) {
  if (p.type != SI_GGML_TYPE_Q4_K || p.cols / 256 > kTcMaxBlocks || (reinterpret_cast<uintptr_t>(p.x) & 15))
    return false;
  if (p.xmode == XM_GATED && p.head_dim != 64 && p.head_dim != 128 && p.head_dim != 256) return false;
  if ((p.xmode == XM_RMS1P || p.xmode == XM_GATED) && !p.xw) return false;
  if ((p.xmode == XM_GATED || p.xmode == XM_SIGGATE) && !p.xaux) return false;
  if (p.pair && (p.nseg != 2 || p.seg[0].rows != p.seg[1].rows)) return false;
  // measured on B200: the tensor-core kernel wins from about 4096 rows of one
  // matrix (17408 x 5120: 13.0 vs 17.2 us; 1024 rows: 5.4 vs 4.6 us), so a
  // grouped call goes there (one launch per segment) only when every segment
  // is that large; otherwise the CUDA-core kernel serves it in one launch
  for (uint32_t i = 0; i < p.nseg; ++i)
    if (p.seg[i].rows < 4096) return false;
  for (uint32_t i = 0; i < p.nseg; ++i)
    if ((reinterpret_cast<uintptr_t>(p.seg[i].w) & 15)) return false;
  return true;
}

static int launch_qmv_tc_seg(const QmvParams& p, uint32_t seg, int seg2, cudaStream_t stream, int sm_count, bool pdl,
                             std::string* msg);

static uint32_t tc_smem_bytes(uint32_t nblk) {
  return kTcRingBytes + nblk * 1024 + nblk * 8 * 4 + ((nblk + 1) & ~1u) * 4 + 2 * kTcMaxStages * 8 + nblk * 8;
}

// CTAs of one launch over `rows` rows (0: the shape does not fit): up to
// kTcCtasPerSm per SM as shared memory allows, at most kTcGroups virtual
// 16-row groups each (a SwiGLU pair stages gate and up groups alike)
static uint32_t tc_grid(uint32_t rows, uint32_t nblk, uint32_t mats, int sm_count, uint32_t* resident = nullptr) {
  static int smem_per_sm = 0;
  if (smem_per_sm == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  }
  const uint32_t ngroups = (rows + 15) / 16;
  const uint32_t fit = std::max(1u, std::min<uint32_t>(kTcCtasPerSm, uint32_t(smem_per_sm) / (tc_smem_bytes(nblk) + 1024)));
  uint32_t nctas = std::min<uint32_t>(ngroups, uint32_t(sm_count) * fit);
  if (resident) *resident = uint32_t(sm_count) * fit;
  while ((ngroups + nctas - 1) / nctas * mats > uint32_t(kTcGroups)) ++nctas;
  return nctas > ngroups ? 0u : nctas;
}

int launch_qmv_tc(const QmvParams& p, cudaStream_t stream, int sm_count, bool pdl, std::string* msg) {
  // every launch must fit before anything is launched (the caller may fall back)
  const uint32_t mats = p.pair ? 2 : 1;
  for (uint32_t i = 0; i < (p.pair ? 1u : p.nseg); ++i)
    if (tc_grid(p.seg[i].rows, p.cols / 256, mats, sm_count) == 0) return SI_E_UNSUPPORTED;
  // segments of a grouped call two to a launch (they share x and its
  // prologue); a SwiGLU pair or a peer exchange is one launch of one matrix
  const uint32_t nl = p.pair ? 1u : p.nseg, step = (p.pair || p.peer.n) ? 1u : 2u;
  for (uint32_t i = 0; i < nl; i += step)
    if (int rc = launch_qmv_tc_seg(p, i, step == 2 && i + 1 < nl ? int(i + 1) : -1, stream, sm_count, pdl, msg))
      return rc;
  return SI_OK;
}

// The band maps of one matrix split over `nctas` CTAs: boxes of the largest
// band (16 ngmax rows) and of the one below it.
static bool tc_band_maps(CUtensorMap* hi, CUtensorMap* lo, const uint8_t* w, uint32_t rows, uint32_t nblk,
                         uint32_t nctas) {
  const uint32_t ngroups = (rows + 15) / 16, ngmax = (ngroups + nctas - 1) / nctas;
  const uint32_t lo_band = 16 * (ngmax > 1 ? ngmax - 1 : 1);
  return q4k_band_map(hi, w, rows, nblk, 16 * ngmax) && q4k_band_map(lo, w, rows, nblk, lo_band);
}

static int launch_qmv_tc_seg(const QmvParams& p, uint32_t seg, int seg2, cudaStream_t stream, int sm_count, bool pdl,
                             std::string* msg) {
  const uint32_t rows = p.seg[seg].rows, nblk = p.cols / 256, mats = p.pair ? 2 : 1;
  const uint32_t ngroups = (rows + 15) / 16;
  const uint32_t smem = tc_smem_bytes(nblk);
  uint32_t resident = 0, nctas = 0, nctas0 = 0, rows1 = 0, ngroups1 = 0;
  if (seg2 < 0) {
    nctas = tc_grid(rows, nblk, mats, sm_count, &resident);
    // every CTA of a peer exchange waits for the other ranks' rows: the whole
    // grid must be resident at once
    if (nctas == 0 || (p.peer.n && nctas > resident)) return SI_E_UNSUPPORTED;
  } else {
    // the grid of the two segments' rows together, shared in proportion to
    // their row groups, each segment at most kTcGroups groups per CTA
    rows1 = p.seg[seg2].rows;
    ngroups1 = (rows1 + 15) / 16;
    const uint32_t total = tc_grid(rows + rows1, nblk, 1, sm_count, &resident);
    if (total < 2) return SI_E_UNSUPPORTED;
    nctas0 = uint32_t((uint64_t(total) * ngroups + (ngroups + ngroups1) / 2) / (ngroups + ngroups1));
    nctas0 = std::min(std::max(nctas0, (ngroups + kTcGroups - 1) / uint32_t(kTcGroups)), ngroups);
    nctas0 = std::max(nctas0, 1u);
    uint32_t nctas1 = total > nctas0 ? total - nctas0 : 1u;
    nctas1 = std::min(std::max(nctas1, (ngroups1 + kTcGroups - 1) / uint32_t(kTcGroups)), ngroups1);
    nctas = nctas0 + std::max(nctas1, 1u);
  }
  CUtensorMap hi, lo, uhi, ulo;
  if (!tc_band_maps(&hi, &lo, p.seg[seg].w, rows, nblk, nctas0 ? nctas0 : nctas)) return SI_E_UNSUPPORTED;
  if (seg2 >= 0) {
    if (!tc_band_maps(&uhi, &ulo, p.seg[seg2].w, rows1, nblk, nctas - nctas0)) return SI_E_UNSUPPORTED;
  } else if (mats == 2) {
    const uint32_t ngmax = (ngroups + nctas - 1) / nctas;
    const uint32_t lo_band = 16 * (ngmax > 1 ? ngmax - 1 : 1);
    if (!q4k_band_map(&uhi, p.seg[1].w, rows, nblk, 16 * ngmax) || !q4k_band_map(&ulo, p.seg[1].w, rows, nblk, lo_band))
      return SI_E_UNSUPPORTED;
  } else {
    uhi = hi;
    ulo = lo;
  }
  static std::atomic<uint32_t> smem_limit[kMaxDevices];
  if (cudaError_t e = raise_smem_limit(qmv_tc_kernel, smem, smem_limit)) {
    if (msg) *msg = std::string("cudaFuncSetAttribute(qmv_tc): ") + cudaGetErrorString(e);
    return SI_E_CUDA;
  }
  TcArgs a = {};
  a.x = p.x;
  a.y = p.seg[seg].y;
  a.resid = p.seg[seg].resid;
  a.xw = p.xw;
  a.xaux = p.xaux;
  a.eps = p.eps;
  a.xmode = p.xmode;
  a.head_dim = p.head_dim;
  a.rows = rows;
  a.nblk = nblk;
  a.ngroups = ngroups;
  a.nctas = nctas;
  a.mats = mats;
  if (seg2 >= 0) {
    a.nctas0 = nctas0;
    a.rows1 = rows1;
    a.ngroups1 = ngroups1;
    a.y1 = p.seg[seg2].y;
    a.resid1 = p.seg[seg2].resid;
  }
  a.err = p.err;
  a.peer = p.peer;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nctas);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qmv_tc_kernel, hi, lo, uhi, ulo, a);
  if (e != cudaSuccess) {
    if (msg) *msg = std::string("qmv_tc launch: ") + cudaGetErrorString(e);
    return SI_E_CUDA;
  }
  return SI_OK;
}

}  // namespace si
