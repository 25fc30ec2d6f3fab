// Batched K-quant matvec: Y[k] = W X[k] for k < batch <= 8, every weight
// super-block read once for all candidates (src/metal.rs:1055-1267
// si_q{4,5,6}_k_matmul_many, 4067-4230 gguf_quant_matmul_many_*; the
// verifier's weight traversal, qwen35_runtime.rs:879-1289).
//
// CUDA-core form for all three types: a warp owns two rows; lane l dequantises
// elements 8l..8l+7 of each 256-column super-block of both rows with the
// reference formulas (quant.rs:18-174), multiplies them by the batch's inputs
// (read through L1 from global memory, [batch][ldx]) and keeps one fp32
// partial sum per (row, candidate); warp sums finish each dot product. Q4_K
// batches of 2..8 go to the tensor-core form (qmatmul_many_tc.cu) when the
// caller supplies its scratch; a batch of one is a plain matvec.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "qmatvec.cuh"

namespace si {

namespace {

// Weight loads: read-only path, L2 evict-first (the weights stream through
// once; the inputs and activations keep the L2).
__device__ __forceinline__ uint32_t ldw_u16(const uint8_t* p, uint64_t pol) {
  unsigned short v;
  asm volatile("ld.global.nc.L2::cache_hint.u16 %0, [%1], %2;" : "=h"(v) : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ uint32_t ldw_u8(const uint8_t* p, uint64_t pol) {
  unsigned short v;
  asm volatile("ld.global.nc.L2::cache_hint.u8 %0, [%1], %2;" : "=h"(v) : "l"(p), "l"(pol));
  return v & 255u;
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

// Eight bytes at a 2-byte aligned address (Q6_K super-blocks are 210 B).
__device__ __forceinline__ uint2 ldw8_a2(const uint8_t* p, uint64_t pol) {
  const uint32_t a = ldw_u16(p, pol), b = ldw_u16(p + 2, pol), c = ldw_u16(p + 4, pol), d = ldw_u16(p + 6, pol);
  return make_uint2(a | (b << 16), c | (d << 16));
}

// d, dmin and the 12 packed scale bytes of a Q4_K/Q5_K super-block (16-byte
// aligned), and the 6-bit scale/min pair `index` from them.
__device__ __forceinline__ void k4_header(const uint8_t* blk, uint64_t pol, int index, float* d, float* mn,
                                          uint32_t* sc, uint32_t* m) {
  const uint4 h = ldw_u4(blk, pol);
  uint8_t b[16];
  *reinterpret_cast<uint4*>(b) = h;
  *d = half_bits_to_float(h.x & 0xffffu);
  *mn = half_bits_to_float(h.x >> 16);
  scale_min_k4(index, b + 4, *sc, *m);
}

__device__ __forceinline__ uint32_t byte_at(const uint2& v, int j) {
  return ((j < 4 ? v.x : v.y) >> (8 * (j & 3))) & 255u;
}

// Elements 8*lane .. 8*lane+7 of one super-block, dequantised as deq_elem
// does (explicitly rounded, so each value is the reference's f32).
template <uint32_t TYPE>
__device__ __forceinline__ void deq8(const uint8_t* blk, int lane, float* v, uint64_t pol);

template <>
__device__ __forceinline__ void deq8<SI_GGML_TYPE_Q4_K>(const uint8_t* blk, int lane, float* v, uint64_t pol) {
  const int g = lane >> 3, r0 = (lane & 7) * 8, hi = r0 >> 5, i0 = r0 & 31;
  float d, mn;
  uint32_t sc, m;
  k4_header(blk, pol, 2 * g + hi, &d, &mn, &sc, &m);
  const float d1 = __fmul_rn(d, float(sc)), m1 = __fmul_rn(mn, float(m));
  const uint2 q = ldw_u2(blk + 16 + 32 * g + i0, pol);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t b = byte_at(q, j);
    v[j] = __fsub_rn(__fmul_rn(d1, float(hi ? (b >> 4) : (b & 15u))), m1);
  }
}

template <>
__device__ __forceinline__ void deq8<SI_GGML_TYPE_Q5_K>(const uint8_t* blk, int lane, float* v, uint64_t pol) {
  const int g = lane >> 3, r0 = (lane & 7) * 8, hi = r0 >> 5, i0 = r0 & 31;
  float d, mn;
  uint32_t sc, m;
  k4_header(blk, pol, 2 * g + hi, &d, &mn, &sc, &m);
  const float d1 = __fmul_rn(d, float(sc)), m1 = __fmul_rn(mn, float(m));
  const uint2 h = ldw_u2(blk + 16 + i0, pol);
  const uint2 q = ldw_u2(blk + 48 + 32 * g + i0, pol);
  const int hb = 2 * g + hi;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t b = byte_at(q, j);
    const uint32_t qq = (hi ? (b >> 4) : (b & 15u)) + (((byte_at(h, j) >> hb) & 1u) ? 16u : 0u);
    v[j] = __fsub_rn(__fmul_rn(d1, float(qq)), m1);
  }
}

template <>
__device__ __forceinline__ void deq8<SI_GGML_TYPE_Q6_K>(const uint8_t* blk, int lane, float* v, uint64_t pol) {
  const int half = lane >> 4, w0 = (lane & 15) * 8, m = w0 >> 5, idx0 = w0 & 31;
  const uint2 lo = ldw8_a2(blk + half * 64 + idx0 + ((m & 1) ? 32 : 0), pol);
  const uint2 hq = ldw8_a2(blk + 128 + half * 32 + idx0, pol);
  const int8_t sc = static_cast<int8_t>(ldw_u8(blk + 192 + half * 8 + (idx0 >> 4) + 2 * m, pol));
  const float d = half_bits_to_float(ldw_u16(blk + 208, pol));
  const float ds = __fmul_rn(d, float(sc));
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t lb = byte_at(lo, j);
    const int nib = int(m < 2 ? (lb & 15u) : (lb >> 4));
    const int q = (nib | int(((byte_at(hq, j) >> (2 * m)) & 3u) << 4)) - 32;
    v[j] = __fmul_rn(ds, float(q));
  }
}

constexpr int kQmmWarps = 8;

template <uint32_t TYPE, int NB>
__global__ void __launch_bounds__(kQmmWarps * 32) qmm_kernel(const QmmParams p) {
  const int lane = threadIdx.x & 31;
  const uint32_t r0 = (blockIdx.x * kQmmWarps + (threadIdx.x >> 5)) * 2;
  pdl_launch_dependents();
  if (r0 >= p.rows) return;
  const bool two = r0 + 1 < p.rows;
  constexpr uint32_t bb = block_bytes_of(TYPE);
  const uint32_t nblk = p.cols / 256;
  const uint8_t* w0 = p.w + uint64_t(r0) * nblk * bb;
  const uint8_t* w1 = two ? w0 + uint64_t(nblk) * bb : w0;
  const uint64_t pol = l2_policy_evict_first();
  float acc0[NB], acc1[NB];
#pragma unroll
  for (int k = 0; k < NB; ++k) acc0[k] = acc1[k] = 0.f;
  pdl_wait();
#pragma unroll 2
  for (uint32_t b = 0; b < nblk; ++b) {
    float v0[8], v1[8];
    deq8<TYPE>(w0 + b * bb, lane, v0, pol);
    deq8<TYPE>(w1 + b * bb, lane, v1, pol);
    const uint32_t c0 = b * 256 + lane * 8;
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const float4* xp = reinterpret_cast<const float4*>(p.x + k * p.ldx + c0);
      const float4 a = __ldg(xp), c = __ldg(xp + 1);
      const float xv[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        acc0[k] = fmaf(v0[j], xv[j], acc0[k]);
        acc1[k] = fmaf(v1[j], xv[j], acc1[k]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const float s0 = warp_sum(acc0[k]), s1 = warp_sum(acc1[k]);
    if (lane == 0) {
      float* y = p.y + k * p.ldy;
      const float* rs = p.resid ? p.resid + k * p.ldr : nullptr;
      y[r0] = rs ? rs[r0] + s0 : s0;
      if (two) y[r0 + 1] = rs ? rs[r0 + 1] + s1 : s1;
    }
  }
}

template <uint32_t TYPE>
cudaError_t launch_nb(const QmmParams& p, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.rows + 2 * kQmmWarps - 1) / (2 * kQmmWarps));
  cfg.blockDim = dim3(kQmmWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  switch (p.batch) {
    case 1: return cudaLaunchKernelEx(&cfg, qmm_kernel<TYPE, 1>, p);
    case 2: return cudaLaunchKernelEx(&cfg, qmm_kernel<TYPE, 2>, p);
    case 3: return cudaLaunchKernelEx(&cfg, qmm_kernel<TYPE, 3>, p);
    case 4: return cudaLaunchKernelEx(&cfg, qmm_kernel<TYPE, 4>, p);
    case 5: return cudaLaunchKernelEx(&cfg, qmm_kernel<TYPE, 5>, p);
    case 6: return cudaLaunchKernelEx(&cfg, qmm_kernel<TYPE, 6>, p);
    case 7: return cudaLaunchKernelEx(&cfg, qmm_kernel<TYPE, 7>, p);
    default: return cudaLaunchKernelEx(&cfg, qmm_kernel<TYPE, 8>, p);
  }
}

}  // namespace

int launch_qmm(const QmmParams& p, cudaStream_t s, int sm_count, bool pdl, std::string* msg) {
  if (p.batch == 0 || p.batch > kQmmMaxBatch || p.rows == 0 || p.cols == 0 || p.cols % 256 ||
      p.cols > kQmvMaxCols || (p.ldx % 4) || p.ldx < p.cols || p.ldy < p.rows ||
      (p.resid && p.ldr < p.rows) || (reinterpret_cast<uintptr_t>(p.x) & 15) ||
      (reinterpret_cast<uintptr_t>(p.w) & (p.type == SI_GGML_TYPE_Q6_K ? 1u : 15u))) {
    if (msg) *msg = "batched quantized matvec dimensions are invalid";
    return SI_E_INVALID;
  }
  if (p.batch == 1) {
    // one input: the matvec family (tensor cores for large Q4_K matrices)
    QmvParams q = {};
    q.type = p.type;
    q.cols = p.cols;
    q.nseg = 1;
    q.seg[0] = {p.w, p.y, p.resid, p.rows, 0};
    q.items = p.rows;
    q.xmode = XM_RAW;
    q.x = p.x;
    q.err = p.err;
    q.scratch = p.qscratch;
    q.scratch_bytes = p.qscratch_bytes;
    return launch_qmv(q, s, sm_count, pdl, msg);
  }
  if (qmm_tc_eligible(p)) {
    const int rc = launch_qmm_tc(p, s, sm_count, pdl, msg);
    if (rc != SI_E_UNSUPPORTED) return rc;
  }
  cudaError_t e;
  switch (p.type) {
    case SI_GGML_TYPE_Q4_K: e = launch_nb<SI_GGML_TYPE_Q4_K>(p, s, pdl); break;
    case SI_GGML_TYPE_Q5_K: e = launch_nb<SI_GGML_TYPE_Q5_K>(p, s, pdl); break;
    case SI_GGML_TYPE_Q6_K: e = launch_nb<SI_GGML_TYPE_Q6_K>(p, s, pdl); break;
    default:
      if (msg) *msg = "unsupported batched quantized weight type";
      return SI_E_UNSUPPORTED;
  }
  if (e != cudaSuccess) {
    if (msg) *msg = std::string("batched matvec launch: ") + cudaGetErrorString(e);
    return SI_E_CUDA;
  }
  return SI_OK;
}

}  // namespace si
