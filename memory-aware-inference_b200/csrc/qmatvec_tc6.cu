// Q6_K matvec y = W x on the tensor cores with exact integer group sums.
//
// Same contract as qmv_kernel<Q6_K> (src/metal.rs:770-1050, 3923 in the
// reference): fp32 y[r] = sum_i w_ri x_i with w = d * sc_G * (q - 32)
// (quant.rs:127-174), the x transforms and the residual epilogue of the other
// matvec kernels.
//
// x as integers (the scheme of qmv_tc_kernel): per 256-column block b, x is
// scaled by 2^(21-e_b) (e_b = exponent of the block's largest |x|) and rounded,
// X = rint(x 2^(21-e_b)), split into three signed base-256 digits.
//
// A Q6_K super-block (210 B: ql[128], qh[64], int8 sc[16], f16 d) holds its
// 256 quants as 8 chunks of 32: element hf*128 + m*32 + i (hf 0..1, m 0..3,
// i 0..31) is the m>>1 nibble of ql[hf*64 + (m&1)*32 + i] with bits 2m, 2m+1
// of qh[hf*32 + i] on top, and its scale is sc[hf*8 + 2m + (i >= 16)]. One
// mma.m16n8k32 (u8 x s8 -> s32) takes a chunk of 16 rows: A = the 6-bit
// quants (0..63), assembled in registers from one ql and one qh word per
// row and k half; B = the digit planes of x, planes 0-2 of the chunk's first
// 16 elements in columns 0-2 and those of the last 16 in columns 4-6 (zero
// elsewhere), so the C fragment separates the two scale groups: lanes
// c = 0, 1 hold the first group's planes, c = 2, 3 the second's. The int8
// scales are applied in integers per MMA; per block the planes are combined
// in fp32, and the -32 offset is 32 * sum_G sc_G * (sum of x over group G).
//
// Data movement. A stage is one 32-row group times a chunk of 8 super-blocks
// (1,680 B, the shortest run of blocks that is a multiple of 16 bytes).
// Tensor-map TMA moves it with 8-byte elements: when a row is a multiple of
// 16 bytes long one box {210 elements, 32 rows} does; when it is 8 mod 16 (20
// or 68 blocks: 5,120 and 17,408 columns) the even rows come from a map with
// a 2-row stride and the odd rows from a map based 8 bytes before row 1 (so
// every box starts 16-byte aligned), box {212 elements, 16 rows}, the odd
// rows landing 8 bytes into their 1,696-byte lines. Sixteen consumer warps:
// half h (warps 8h..8h+7) takes rows 16h..16h+15 of the group, and slot w of
// a half owns block w of every chunk, so a warp's 2-byte misalignment (block
// w starts 210 w bytes into the chunk) is fixed: one funnel shift per 4-byte
// quant word. The digits of all of x are made once per CTA before the first
// stage is read. One CTA per SM holds three stages (162 KB) and the digits.
//
// Work split. The (group, chunk) units are dealt out evenly, a contiguous
// range per CTA. A group inside one CTA's range is summed there: per row,
// each slot's chunks in chunk order, then the slots in slot order. A group
// that straddles CTAs is finished by the last of them to arrive (a counter
// per group): its first CTA leaves its slots' prefix sums, the others each
// chunk's contribution, and the finisher continues every slot's sum in chunk
// order before adding the slots. Every row's arithmetic is therefore the same
// whatever the grid, the row sharding or the CTA count. The counters and
// partial sums live in the launching stream's slot of the context's scratch;
// without one the CTAs take whole groups.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <type_traits>
#include <string>

#include "common.cuh"
#include "qmatvec.cuh"
#include "peer_exchange.cuh"

namespace si {

namespace {

constexpr int kT6Slots = 8;                    // warps per 16-row half: slot w owns block w of every chunk
constexpr int kT6Warps = 2 * kT6Slots;         // consumer warps: halves 0 and 1 of a 32-row group
constexpr int kT6Threads = (kT6Warps + 1) * 32;
constexpr int kT6Stages = 3;
constexpr uint32_t kT6EvenLine = 1680;         // 8 blocks of an even (or 16-byte aligned) row
constexpr uint32_t kT6OddLine = 1696;          // 8 blocks of an odd row, 8 bytes in
constexpr uint32_t kT6StageBytes = 16 * kT6EvenLine + 16 * kT6OddLine;  // 54,016 (32 aligned rows: 53,760)
constexpr uint32_t kT6StagePitch = 54016;      // 128-byte multiple
constexpr uint32_t kT6MaxBlocks = 72;
constexpr int kT6DigPerWarp = (kT6MaxBlocks + kT6Warps - 1) / kT6Warps;  // blocks of x per warp's digits
constexpr uint32_t kT6DigBlock = 8 * 96;       // per block: 8 chunks x 3 planes x 32 s8 digits

struct T6Args {
  const float* x;
  float* y;
  const float* resid;
  const float* xw;
  const float* xaux;
  float eps;
  int xmode;
  uint32_t head_dim;
  uint32_t rows, nblk, ngroups, nctas, nchunks;
  uint32_t paired;   // 1: even / odd row maps (rows 8 mod 16 bytes long), 0: one map
  uint32_t split;    // 1: CTAs own ranges of (group, chunk) units; 0: ranges of whole groups
  // split: per group shared by CTAs, indexed by the group's first CTA (a CTA
  // heads at most one shared group: the last of its range)
  uint32_t* counters;  // [nctas] CTAs finished with the group (zero between launches)
  float* part;       // [nctas][16 warps][nchunks + 1][16] the head's sums, the others' contributions
  int* err;
  PeerOut peer;      // n > 0: the rows are gathered into every rank's vector (peer_exchange.cuh)
};

// CTA holding unit u under the even split of U units over G CTAs.
__device__ __forceinline__ uint32_t t6_cta_of(uint32_t u, uint32_t U, uint32_t G) {
  return uint32_t((uint64_t(u + 1) * G - 1) / U);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void mma_u8s8(int* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// Four bytes at `p` + off of a row whose bytes start `sh` / 8 bytes past a
// 4-byte boundary (sh = 0 or 16; off a multiple of 4).
__device__ __forceinline__ uint32_t ld_row32(const uint8_t* aligned, uint32_t off, uint32_t sh) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(aligned + off);
  return __funnelshift_r(w[0], w[1], sh);
}

// 6-bit quants of four consecutive elements: low or high nibbles of `l`,
// bits 2m, 2m+1 of `h` as bits 4, 5.
template <int M>
__device__ __forceinline__ uint32_t q6_word(uint32_t l, uint32_t h) {
  const uint32_t lo = (M >> 1) ? ((l >> 4) & 0x0F0F0F0Fu) : (l & 0x0F0F0F0Fu);
  const uint32_t hi = M == 0 ? ((h << 4) & 0x30303030u)
                      : M == 1 ? ((h << 2) & 0x30303030u)
                      : M == 2 ? (h & 0x30303030u)
                               : ((h >> 2) & 0x30303030u);
  return lo | hi;
}

// prmt selector that moves byte k (0..3) of a word into byte 0 and fills the
// other bytes with its sign (PTX prmt.b32: a selector nibble's bit 3
// replicates the sign of the byte its bits 2:0 choose).
__host__ __device__ constexpr uint32_t sx_sel(uint32_t k) {
  return k | ((k | 8u) << 4) | ((k | 8u) << 8) | ((k | 8u) << 12);
}

// The sign-extended byte that `sel` (an sx_sel value) picks from a word.
__device__ __forceinline__ int sbyte_p(uint32_t w, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
  return int(r);
}

__global__ void __launch_bounds__(kT6Threads, 1)
    qmv_tc6_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
                   const __grid_constant__ T6Args a) {
  extern __shared__ __align__(128) uint8_t tsm[];
  uint8_t* ring = tsm;
  uint8_t* xd = ring + kT6Stages * kT6StagePitch;                   // [blk][8 chunks][3 planes][32] s8
  float* xs16 = reinterpret_cast<float*>(xd + a.nblk * kT6DigBlock);  // [blk][16] group sums of x
  float* escale = xs16 + a.nblk * 16;                                // [blk] 2^(e-21)
  float* red = escale + ((a.nblk + 3) & ~3u);                        // [16 warps][16 rows]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + kT6Warps * 16);
  uint64_t* empty = full + kT6Stages;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this CTA's units (group, chunk), group-major: a range of whole groups, or
  // (split) an even share of all units, whose first and last groups may be
  // shared with the neighbouring CTAs
  const uint32_t U = a.ngroups * a.nchunks;
  uint32_t u0, u1;
  if (a.split) {
    u0 = uint32_t(uint64_t(blockIdx.x) * U / a.nctas);
    u1 = uint32_t(uint64_t(blockIdx.x + 1) * U / a.nctas);
  } else {
    u0 = uint32_t(uint64_t(blockIdx.x) * a.ngroups / a.nctas) * a.nchunks;
    u1 = uint32_t(uint64_t(blockIdx.x + 1) * a.ngroups / a.nctas) * a.nchunks;
  }
  const uint32_t nst = u1 - u0;                                      // stages of this CTA
  __shared__ uint32_t s_last;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kT6Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kT6Warps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kT6Warps) {
    // ---- producer: per stage, the chunk's box(es) of one 16-row group ----
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      for (uint32_t t = 0; t < nst; ++t) {
        const uint32_t s = t % kT6Stages, grp = (u0 + t) / a.nchunks, ch = (u0 + t) % a.nchunks;
        if (t >= uint32_t(kT6Stages) && !mbar_wait_bounded(&empty[s], ((t / kT6Stages) - 1) & 1)) {
          if (a.err) atomicOr(a.err, KERR_TIMEOUT_EMPTY);
          break;
        }
        uint8_t* dst = ring + s * kT6StagePitch;
        if (a.paired) {
          mbar_arrive_expect_tx(&full[s], kT6StageBytes);
          tma_load_2d(smem_u32(dst), &map0, int(ch * 210), int(grp * 16), &full[s], pol);
          tma_load_2d(smem_u32(dst + 16 * kT6EvenLine), &map1, int(ch * 210), int(grp * 16), &full[s], pol);
        } else {
          mbar_arrive_expect_tx(&full[s], 32 * kT6EvenLine);
          tma_load_2d(smem_u32(dst), &map0, int(ch * 210), int(grp * 32), &full[s], pol);
        }
      }
    }
    return;
  }

  // ---- consumers ----
  pdl_wait();
  // the launch's epoch of the peer exchange (the previous grid has finished)
  __shared__ uint32_t s_epoch;
  if (a.peer.n && threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(a.peer.epoch) + 1;
  float rms_inv = 1.f;
  if (a.xmode == XM_RMS1P) {
    // (1+w) RMSNorm over the whole vector (qwen35.rs:53-86, heads = 1)
    __shared__ float s_red[kT6Warps];
    float ss = 0.f;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    for (uint32_t i = threadIdx.x; i < a.nblk * 64; i += kT6Warps * 32) {
      const float4 u = x4[i];
      ss += u.x * u.x + u.y * u.y + u.z * u.z + u.w * u.w;
    }
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    asm volatile("bar.sync 1, %0;" ::"r"(kT6Warps * 32) : "memory");
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kT6Warps; ++w) tot += s_red[w];
    rms_inv = 1.0f / sqrtf(tot / float(a.nblk * 256) + a.eps);
  }
  // ---- digits of x, all blocks, before the first stage is read ----
  // (every load of this warp's blocks of x leaves before the first is used)
  float4 xr[kT6DigPerWarp][2];
#pragma unroll
  for (int j = 0; j < kT6DigPerWarp; ++j) {
    const uint32_t b = uint32_t(warp) + j * kT6Warps;
    if (b < a.nblk) {
      const float4* xp = reinterpret_cast<const float4*>(a.x + b * 256 + lane * 8);
      xr[j][0] = xp[0];
      xr[j][1] = xp[1];
    }
  }
#pragma unroll
  for (int j = 0; j < kT6DigPerWarp; ++j) {
    const uint32_t b = uint32_t(warp) + j * kT6Warps;
    if (b >= a.nblk) break;
    float v[8];
    const uint32_t e0 = b * 256 + lane * 8;
    v[0] = xr[j][0].x; v[1] = xr[j][0].y; v[2] = xr[j][0].z; v[3] = xr[j][0].w;
    v[4] = xr[j][1].x; v[5] = xr[j][1].y; v[6] = xr[j][1].z; v[7] = xr[j][1].w;
    if (a.xmode == XM_RMS1P) {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = v[k] * rms_inv * (1.0f + a.xw[e0 + k]);
    } else if (a.xmode == XM_GATED) {
      // per head of head_dim: x * rsqrt(mean x^2 + eps) * w[d] * SiLU(z) (qwen35.rs:14-49)
      const uint32_t hl = a.head_dim / 8;
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
    float mx = 0.f, sum = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      mx = fmaxf(mx, fabsf(v[k]));
      sum += v[k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // the 16-element group of lanes 2j, 2j+1
    int e = int((__float_as_uint(mx) >> 23) & 255u) - 127;
    e = max(e, -100);
    const float up = __uint_as_float(uint32_t(21 - e + 127) << 23);  // 2^(21-e), exact
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
    // lane l: elements 8l..8l+7 = chunk l / 4 (hf * 4 + m), i = (l % 4) * 8 ..
    uint8_t* dst = xd + b * kT6DigBlock + (uint32_t(lane) >> 2) * 96 + (uint32_t(lane) & 3) * 8;
#pragma unroll
    for (int p = 0; p < 3; ++p) *reinterpret_cast<uint2*>(dst + p * 32) = make_uint2(pl[p][0], pl[p][1]);
    if ((lane & 1) == 0) xs16[b * 16 + (uint32_t(lane) >> 1)] = sum;
    if (lane == 0) escale[b] = __uint_as_float(uint32_t(e - 21 + 127) << 23);  // 2^(e-21)
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kT6Warps * 32) : "memory");

  const uint32_t g = uint32_t(lane) >> 2, c = uint32_t(lane) & 3;
  const uint32_t hi = c >> 1;                            // lanes 2, 3: the chunk's second scale group
  // scale byte of an even / odd m inside its word, as prmt selectors
  const uint32_t sel0 = sx_sel(hi), sel1 = sx_sel(2 + hi);
  const uint32_t slot = uint32_t(warp) % kT6Slots, half = uint32_t(warp) / kT6Slots;
  // this warp's block inside a chunk starts 210 slot bytes in: 2-byte aligned for odd slots
  const uint32_t boff8 = slot * 210;
  const uint32_t bal = boff8 & ~3u, sh = (boff8 & 2) * 8;
  // rows g and g+8 of this half of the group (stage rows r0 = 16 half + g and
  // r0 + 8): even rows in the first 16 lines, odd rows (paired maps) in the
  // next 16, 8 bytes in
  const uint32_t sr0 = half * 16 + g, sr8 = sr0 + 8;
  const uint32_t line0 = a.paired ? ((sr0 & 1) ? 16 * kT6EvenLine + (sr0 >> 1) * kT6OddLine + 8 : (sr0 >> 1) * kT6EvenLine)
                                  : sr0 * kT6EvenLine;
  const uint32_t line8 = a.paired ? ((sr8 & 1) ? 16 * kT6EvenLine + (sr8 >> 1) * kT6OddLine + 8 : (sr8 >> 1) * kT6EvenLine)
                                  : sr8 * kT6EvenLine;
  // B fragment: lane (g, c) holds B[k = 4c..4c+3][g] and B[16+4c..][g]
  const bool b_lo = g < 3, b_hi = g >= 4 && g < 7;
  const uint32_t boff = b_lo ? g * 32 + 4 * c : (b_hi ? (g - 4) * 32 + 16 + 4 * c : 0);
  float yg = 0.f, yg8 = 0.f;
  bool alive = true;
  for (uint32_t t = 0; t < nst; ++t) {
    const uint32_t s = t % kT6Stages, ch = (u0 + t) % a.nchunks, grp = (u0 + t) / a.nchunks;
    // this CTA's chunks of the group: [cs, ce)
    const uint32_t cs = u0 > grp * a.nchunks ? u0 - grp * a.nchunks : 0;
    const uint32_t ce = min(a.nchunks, u1 - grp * a.nchunks);
    const bool whole = cs == 0 && ce == a.nchunks, head = cs == 0;
    const uint32_t b = ch * kT6Slots + slot;           // this warp's block
    const bool has = b < a.nblk;
    // a wait that ran out stops this warp's arithmetic, not its barriers
    if (alive && !mbar_wait_bounded(&full[s], (t / kT6Stages) & 1)) {
      if (a.err) atomicOr(a.err, KERR_TIMEOUT_FULL);
      alive = false;
    }
    // the stage's arithmetic, for a slot whose rows start 4-byte aligned
    // (even slots: one shared load per word) or 2 bytes past (odd slots)
    auto stage_math = [&](auto aligned) {
      constexpr bool AL = decltype(aligned)::value;
      auto LD = [&](const uint8_t* r, uint32_t off) -> uint32_t {
        if constexpr (AL) return *reinterpret_cast<const uint32_t*>(r + off);
        else return ld_row32(r, off, 16);
      };
        const uint8_t* r0 = ring + s * kT6StagePitch + line0 + bal;
        const uint8_t* r8 = ring + s * kT6StagePitch + line8 + bal;
        uint32_t sw0[4], sw8[4];
  #pragma unroll
        for (int k = 0; k < 4; ++k) {
          sw0[k] = LD(r0, 192 + 4 * k);
          sw8[k] = LD(r8, 192 + 4 * k);
        }
        const float d0 = half_bits_to_float(LD(r0, 208));
        const float d8 = half_bits_to_float(LD(r8, 208));
        int acc[4] = {0, 0, 0, 0};
        const uint8_t* xb = xd + b * kT6DigBlock + boff;
  #pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t l0[2][2], l8[2][2], h0[2], h8[2];
  #pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            h0[kk] = LD(r0, 128 + hf * 32 + 16 * kk + 4 * c);
            h8[kk] = LD(r8, 128 + hf * 32 + 16 * kk + 4 * c);
  #pragma unroll
            for (int mm = 0; mm < 2; ++mm) {
              l0[mm][kk] = LD(r0, hf * 64 + mm * 32 + 16 * kk + 4 * c);
              l8[mm][kk] = LD(r8, hf * 64 + mm * 32 + 16 * kk + 4 * c);
            }
          }
  #pragma unroll
          for (int m = 0; m < 4; ++m) {
            uint32_t A[4];
            if (m == 0) {
              A[0] = q6_word<0>(l0[0][0], h0[0]); A[1] = q6_word<0>(l8[0][0], h8[0]);
              A[2] = q6_word<0>(l0[0][1], h0[1]); A[3] = q6_word<0>(l8[0][1], h8[1]);
            } else if (m == 1) {
              A[0] = q6_word<1>(l0[1][0], h0[0]); A[1] = q6_word<1>(l8[1][0], h8[0]);
              A[2] = q6_word<1>(l0[1][1], h0[1]); A[3] = q6_word<1>(l8[1][1], h8[1]);
            } else if (m == 2) {
              A[0] = q6_word<2>(l0[0][0], h0[0]); A[1] = q6_word<2>(l8[0][0], h8[0]);
              A[2] = q6_word<2>(l0[0][1], h0[1]); A[3] = q6_word<2>(l8[0][1], h8[1]);
            } else {
              A[0] = q6_word<3>(l0[1][0], h0[0]); A[1] = q6_word<3>(l8[1][0], h8[0]);
              A[2] = q6_word<3>(l0[1][1], h0[1]); A[3] = q6_word<3>(l8[1][1], h8[1]);
            }
            const uint32_t bw = (b_lo || b_hi) ? *reinterpret_cast<const uint32_t*>(xb + (hf * 4 + m) * 96) : 0u;
            int C[4];
            mma_u8s8(C, A, b_lo ? bw : 0u, b_hi ? bw : 0u);
            // scale sc[hf * 8 + 2m + hi]: word hf * 2 + m / 2, byte (m & 1) * 2 + hi
            const uint32_t wsel = hf * 2 + (m >> 1), bsel = (m & 1) ? sel1 : sel0;
            const int s0 = sbyte_p(sw0[wsel], bsel), s8 = sbyte_p(sw8[wsel], bsel);
            acc[0] += s0 * C[0];
            acc[1] += s0 * C[1];
            acc[2] += s8 * C[2];
            acc[3] += s8 * C[3];
          }
        }
        // digit columns: lanes c = 0, 2 hold planes 0 and 1, lanes c = 1, 3 plane 2
        float f0 = (c & 1) ? 65536.f * float(acc[0]) : fmaf(256.f, float(acc[1]), float(acc[0]));
        float f8 = (c & 1) ? 65536.f * float(acc[2]) : fmaf(256.f, float(acc[3]), float(acc[2]));
        f0 += __shfl_xor_sync(0xffffffffu, f0, 1);
        f8 += __shfl_xor_sync(0xffffffffu, f8, 1);
        f0 += __shfl_xor_sync(0xffffffffu, f0, 2);
        f8 += __shfl_xor_sync(0xffffffffu, f8, 2);
        // -32 offset: lane c takes groups 4c..4c+3 (scale word c)
        const float4 xg = *reinterpret_cast<const float4*>(xs16 + b * 16 + 4 * c);
        const uint32_t w0c = c == 0 ? sw0[0] : c == 1 ? sw0[1] : c == 2 ? sw0[2] : sw0[3];
        const uint32_t w8c = c == 0 ? sw8[0] : c == 1 ? sw8[1] : c == 2 ? sw8[2] : sw8[3];
        float mt0 = float(sbyte_p(w0c, sx_sel(0))) * xg.x + float(sbyte_p(w0c, sx_sel(1))) * xg.y;
        mt0 += float(sbyte_p(w0c, sx_sel(2))) * xg.z + float(sbyte_p(w0c, sx_sel(3))) * xg.w;
        float mt8 = float(sbyte_p(w8c, sx_sel(0))) * xg.x + float(sbyte_p(w8c, sx_sel(1))) * xg.y;
        mt8 += float(sbyte_p(w8c, sx_sel(2))) * xg.z + float(sbyte_p(w8c, sx_sel(3))) * xg.w;
        mt0 += __shfl_xor_sync(0xffffffffu, mt0, 1);
        mt8 += __shfl_xor_sync(0xffffffffu, mt8, 1);
        mt0 += __shfl_xor_sync(0xffffffffu, mt0, 2);
        mt8 += __shfl_xor_sync(0xffffffffu, mt8, 2);
        const float es = escale[b];
        const float c0 = d0 * fmaf(-32.f, mt0, es * f0), c8 = d8 * fmaf(-32.f, mt8, es * f8);
        yg += c0;
        yg8 += c8;
        if (!head && c == 0) {
          // a later CTA finishes this group: keep the contribution itself
          const uint32_t hc = t6_cta_of(grp * a.nchunks, U, a.nctas);
          float* pp = a.part + ((uint64_t(hc) * kT6Warps + warp) * (a.nchunks + 1) + 1 + ch) * 16;
          pp[g] = c0;
          pp[g + 8] = c8;
        }
    };
    if (has && alive) {
      if (sh == 0)
        stage_math(std::true_type{});
      else
        stage_math(std::false_type{});
    } else if (!head && c == 0) {
      const uint32_t hc = t6_cta_of(grp * a.nchunks, U, a.nctas);
      float* pp = a.part + ((uint64_t(hc) * kT6Warps + warp) * (a.nchunks + 1) + 1 + ch) * 16;
      pp[g] = 0.f;
      pp[g + 8] = 0.f;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (ch == ce - 1) {
      // ---- the group's last chunk in this CTA: the warps' sums, in warp order ----
      if (whole) {
        if (c == 0) {
          red[warp * 16 + g] = yg;
          red[warp * 16 + g + 8] = yg8;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kT6Warps * 32) : "memory");
      } else {
        if (head && c == 0) {
          float* pp = a.part + (uint64_t(blockIdx.x) * kT6Warps + warp) * (a.nchunks + 1) * 16;
          pp[g] = yg;
          pp[g + 8] = yg8;
        }
        // every partial of this CTA precedes the group's counter (barrier + one fence)
        asm volatile("bar.sync 1, %0;" ::"r"(kT6Warps * 32) : "memory");
        if (threadIdx.x == 0) {
          __threadfence();
          const uint32_t c_first = t6_cta_of(grp * a.nchunks, U, a.nctas);
          const uint32_t c_last = t6_cta_of(grp * a.nchunks + a.nchunks - 1, U, a.nctas);
          const uint32_t old = atomicAdd(&a.counters[c_first], 1u);
          const bool last = old + 1 == c_last - c_first + 1;
          if (last) {
            a.counters[c_first] = 0;  // ready for the next launch
            __threadfence();
          }
          s_last = last ? 1u : 0u;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kT6Warps * 32) : "memory");
        if (s_last && threadIdx.x < kT6Warps * 16) {
          // thread j: row j % 16 of warp j / 16's sum: the head's prefix, then
          // the other CTAs' contributions in chunk order (loads first)
          const uint32_t row = threadIdx.x & 15, wj = threadIdx.x >> 4;
          const uint32_t c_head = t6_cta_of(grp * a.nchunks, U, a.nctas);
          const uint32_t head_end = min(a.nchunks, uint32_t(uint64_t(c_head + 1) * U / a.nctas) - grp * a.nchunks);
          const float* pp = a.part + (uint64_t(c_head) * kT6Warps + wj) * (a.nchunks + 1) * 16 + row;
          float v[10];
          float S = __ldcg(pp);
#pragma unroll
          for (uint32_t k = 0; k < 10; ++k) {
            const uint32_t chk = head_end + k;
            v[k] = chk < a.nchunks ? __ldcg(pp + (1 + chk) * 16) : 0.f;
          }
#pragma unroll
          for (uint32_t k = 0; k < 10; ++k)
            if (head_end + k < a.nchunks) S += v[k];
          red[wj * 16 + row] = S;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kT6Warps * 32) : "memory");
      }
      if ((whole || s_last) && warp == 0) {
        // lane l: row l of the group, the sum over its half's slots in slot order
        const float* rh = red + (uint32_t(lane) >> 4) * kT6Slots * 16 + (lane & 15);
        float tot = rh[0];
#pragma unroll
        for (int w = 1; w < kT6Slots; ++w) tot += rh[w * 16];
        const uint32_t row = grp * 32 + uint32_t(lane);
        if (row < a.rows) {
          const float v = a.resid ? a.resid[row] + tot : tot;
          if (a.peer.n)
            peer_store_row(a.peer, s_epoch, row, v);
          else
            a.y[row] = v;
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kT6Warps * 32) : "memory");
      yg = yg8 = 0.f;
    }
  }
  if (a.peer.n) peer_gather(a.peer, a.nctas, s_epoch, a.err, kT6Warps * 32);
}

}  // namespace

static PFN_cuTensorMapEncodeTiled_v12000 t6_encoder() {
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

// Rows of Q6_K super-blocks as 8-byte elements: `lines` lines of `elems`
// elements `pitch` bytes apart from `base`, box {box_elems, box_lines}.
static bool t6_map(CUtensorMap* m, const void* base, uint64_t elems, uint64_t lines, uint64_t pitch,
                   uint32_t box_elems, uint32_t box_lines) {
  auto enc = t6_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) || (pitch & 15) || lines == 0) return false;
  const cuuint64_t dims[2] = {elems, lines};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {box_elems, box_lines};
  const cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool qmv_tc6_eligible(const QmvParams& p) {
  const uint32_t nblk = p.cols / 256;
  if (p.type != SI_GGML_TYPE_Q6_K || p.pair || p.nseg != 1 || nblk > kT6MaxBlocks || nblk % 4 ||
      (reinterpret_cast<uintptr_t>(p.x) & 15) || p.seg[0].rows < kTc6MinRows ||
      (reinterpret_cast<uintptr_t>(p.seg[0].w) & 15))
    return false;
  if (p.seg[0].rows < kTc6AnyWidthRows && nblk < kTc6WideBlocks) return false;
  if (p.xmode == XM_GATED && p.head_dim != 64 && p.head_dim != 128 && p.head_dim != 256) return false;
  if ((p.xmode == XM_RMS1P || p.xmode == XM_GATED) && !p.xw) return false;
  if ((p.xmode == XM_GATED || p.xmode == XM_SIGGATE) && !p.xaux) return false;
  return true;
}

uint64_t qmv_tc6_scratch_bytes(uint32_t sm_count) {
  // counters (one word per CTA) then the partial sums of the shared groups
  return 4096 + uint64_t(sm_count) * kT6Warps * (kT6MaxBlocks / 8 + 1) * 16 * 4;
}

int launch_qmv_tc6(const QmvParams& p, cudaStream_t stream, int sm_count, bool pdl, std::string* msg) {
  const uint32_t rows = p.seg[0].rows, nblk = p.cols / 256;
  const uint64_t row_bytes = uint64_t(nblk) * 210;  // nblk % 4 == 0: a multiple of 8
  const bool paired = (row_bytes % 16) != 0;         // 8 mod 16
  const uint32_t ngroups = (rows + 31) / 32;
  const uint32_t smem = kT6Stages * kT6StagePitch + nblk * kT6DigBlock + nblk * 16 * 4 + ((nblk + 3) & ~3u) * 4 +
                        kT6Warps * 16 * 4 + 2 * kT6Stages * 8;
  const uint8_t* w = p.seg[0].w;
  CUtensorMap m0, m1;
  if (paired) {
    // even rows: lines 2 rows apart from row 0; odd rows: from 8 bytes before row 1
    if (!t6_map(&m0, w, row_bytes / 8, (rows + 1) / 2, 2 * row_bytes, 210, 16)) return SI_E_UNSUPPORTED;
    if (rows / 2 == 0 || !t6_map(&m1, w + row_bytes - 8, row_bytes / 8 + 1, rows / 2, 2 * row_bytes, 212, 16))
      return SI_E_UNSUPPORTED;
  } else {
    if (!t6_map(&m0, w, row_bytes / 8, rows, row_bytes, 210, 32)) return SI_E_UNSUPPORTED;
    m1 = m0;
  }
  static std::atomic<uint32_t> smem_limit[kMaxDevices];
  if (cudaError_t e = raise_smem_limit(qmv_tc6_kernel, smem, smem_limit)) {
    if (msg) *msg = std::string("cudaFuncSetAttribute(qmv_tc6): ") + cudaGetErrorString(e);
    return SI_E_CUDA;
  }
  T6Args a = {};
  a.x = p.x;
  a.y = p.seg[0].y;
  a.resid = p.seg[0].resid;
  a.xw = p.xw;
  a.xaux = p.xaux;
  a.eps = p.eps;
  a.xmode = p.xmode;
  a.head_dim = p.head_dim;
  a.rows = rows;
  a.nblk = nblk;
  a.ngroups = ngroups;
  a.nchunks = (nblk + 7) / 8;
  a.paired = paired ? 1u : 0u;
  // an even share of the (group, chunk) units per CTA, the groups shared by
  // neighbouring CTAs finished through the scratch of the launching stream;
  // without scratch, whole groups per CTA
  a.nctas = std::min<uint32_t>(ngroups * a.nchunks, uint32_t(sm_count));
  if (p.scratch && qmv_tc6_scratch_bytes(uint32_t(sm_count)) <= p.scratch_bytes && a.nchunks <= 9) {
    a.split = 1;
    a.counters = static_cast<uint32_t*>(p.scratch);
    a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(p.scratch) + 4096);
  } else {
    a.split = 0;
    a.nctas = std::min<uint32_t>(ngroups, uint32_t(sm_count));
  }
  a.err = p.err;
  a.peer = p.peer;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nctas);
  cfg.blockDim = dim3(kT6Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qmv_tc6_kernel, m0, m1, a);
  if (e != cudaSuccess) {
    if (msg) *msg = std::string("qmv_tc6 launch: ") + cudaGetErrorString(e);
    return SI_E_CUDA;
  }
  return SI_OK;
}

}  // namespace si
