// Non-matvec kernels of the batch-1 decode path (sm_100a).
//
// Where the reference fixes an evaluation order (qwen35.rs, metal.rs), the
// per-element arithmetic here follows it with explicitly rounded operations
// (__fmul_rn / __fadd_rn prevent FMA contraction), so the dequant is
// bit-exact and the recurrence/conv match the CPU code to the last ulp of the
// transcendentals. Reductions that the reference runs serially are done as
// parallel trees where that is the only difference (within 1e-5 rel-L2).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"
#include "peer_exchange.cuh"

namespace si {

// ---------------------------------------------------------------------------
// Dequantization (quant.rs:18-174), one thread per output element.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float deq_elem(uint32_t type, const uint8_t* blk, int e) {
  if (type == SI_GGML_TYPE_Q6_K) {
    const int half = e >> 7, w = e & 127, m = w >> 5, idx = w & 31;
    const uint8_t* low = blk + half * 64;
    const uint8_t hb = blk[128 + half * 32 + idx];
    const uint8_t lb = low[idx + ((m & 1) ? 32 : 0)];
    const int nib = (m < 2) ? (lb & 0x0f) : (lb >> 4);
    const int q = (nib | (((hb >> (2 * m)) & 3) << 4)) - 32;
    const int8_t sc = static_cast<int8_t>(blk[192 + half * 8 + (idx >> 4) + 2 * m]);
    const float d = half_bits_to_float(uint32_t(blk[208]) | (uint32_t(blk[209]) << 8));
    return __fmul_rn(__fmul_rn(d, float(sc)), float(q));
  }
  const float d = half_bits_to_float(uint32_t(blk[0]) | (uint32_t(blk[1]) << 8));
  const float mn = half_bits_to_float(uint32_t(blk[2]) | (uint32_t(blk[3]) << 8));
  const int g = e >> 6, r = e & 63, hi = r >> 5, i = r & 31;
  uint32_t sc, m;
  scale_min_k4(2 * g + hi, blk + 4, sc, m);
  int q;
  if (type == SI_GGML_TYPE_Q4_K) {
    const uint8_t b = blk[16 + 32 * g + i];
    q = hi ? (b >> 4) : (b & 0x0f);
  } else {
    const uint8_t b = blk[48 + 32 * g + i];
    const uint8_t h = blk[16 + i];
    q = (hi ? (b >> 4) : (b & 0x0f)) + (((h >> (2 * g + hi)) & 1) ? 16 : 0);
  }
  const float d1 = __fmul_rn(d, float(sc));
  const float m1 = __fmul_rn(mn, float(m));
  return __fsub_rn(__fmul_rn(d1, float(q)), m1);
}

__global__ void dequant_kernel(uint32_t type, const uint8_t* w, uint64_t n, float* out) {
  const uint32_t bb = block_bytes_of(type);
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += uint64_t(gridDim.x) * blockDim.x)
    out[i] = deq_elem(type, w + (i >> 8) * bb, int(i & 255));
}

void launch_dequant(uint32_t type, const uint8_t* w, uint64_t elements, float* out,
                    cudaStream_t s) {
  uint64_t blocks = (elements + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  dequant_kernel<<<unsigned(blocks), 256, 0, s>>>(type, w, elements, out);
}

// ---------------------------------------------------------------------------
// F32 matvec (metal.rs:263-305), one warp per row.
// ---------------------------------------------------------------------------
__global__ void f32_matvec_kernel(const float* w, uint64_t rows, uint64_t cols, const float* x,
                                  float* y) {
  const uint64_t row = uint64_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* wr = reinterpret_cast<const float4*>(w + row * cols);
  const float4* xv = reinterpret_cast<const float4*>(x);
  float acc = 0.f;
  for (uint64_t i = lane; i < cols / 4; i += 32) {
    const float4 a = __ldg(wr + i), b = xv[i];
    acc += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = acc;
}

void launch_f32_matvec(const float* w, uint64_t rows, uint64_t cols, const float* x, float* y,
                       cudaStream_t s) {
  const unsigned blocks = unsigned((rows + 7) / 8);
  f32_matvec_kernel<<<blocks, 256, 0, s>>>(w, rows, cols, x, y);
}

// ---------------------------------------------------------------------------
// Norms (qwen35.rs:14-86): one CTA per head.
// ---------------------------------------------------------------------------
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < int(blockDim.x >> 5); ++i) t += red[i];
  return t;
}

__global__ void rms_norm_kernel(const float* x, const float* z, const float* w, uint32_t hd,
                                float eps, float* out) {
  __shared__ float red[32];
  const uint64_t base = uint64_t(blockIdx.x) * hd;
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) ss += x[base + i] * x[base + i];
  const float tot = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(tot / float(hd) + eps);
  for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
    if (z) {
      const float g = z[base + i];
      out[base + i] = x[base + i] * inv * w[i] * (g / (1.0f + expf(-g)));
    } else {
      out[base + i] = x[base + i] * inv * (1.0f + w[i]);
    }
  }
}

void launch_rms_norm_heads(const float* x, const float* w, uint32_t heads, uint32_t hd,
                           float eps, float* out, cudaStream_t s) {
  rms_norm_kernel<<<heads, 256, 0, s>>>(x, nullptr, w, hd, eps, out);
}

void launch_rms_norm_gated(const float* x, const float* z, const float* w, uint32_t heads,
                           uint32_t hd, float eps, float* out, cudaStream_t s) {
  rms_norm_kernel<<<heads, 256, 0, s>>>(x, z, w, hd, eps, out);
}

// ---------------------------------------------------------------------------
// Causal conv step (qwen35.rs:93-130), one thread per channel, the
// reference's accumulation order, state written to a separate buffer.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float conv_channel(float xin, const float* st, const float* wc,
                                              uint32_t k) {
  float v = __fmul_rn(xin, wc[k - 1]);
  for (uint32_t t = 0; t + 1 < k; ++t) v = __fadd_rn(v, __fmul_rn(st[t], wc[t]));
  return v;
}

__global__ void conv1d_kernel(const float* x, const float* sin, const float* w, uint32_t C,
                              uint32_t k, float* out, float* sout) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float* st = sin + uint64_t(c) * (k - 1);
  const float v = conv_channel(x[c], st, w + uint64_t(c) * k, k);
  out[c] = v / (1.0f + expf(-v));
  float* so = sout + uint64_t(c) * (k - 1);
  for (uint32_t t = 0; t + 2 < k; ++t) so[t] = st[t + 1];
  so[k - 2] = x[c];
}

void launch_conv1d_step(const float* x, const float* state_in, const float* w,
                        uint32_t channels, uint32_t kernel, float* out, float* state_out,
                        cudaStream_t s) {
  conv1d_kernel<<<(channels + 255) / 256, 256, 0, s>>>(x, state_in, w, channels, kernel, out,
                                                        state_out);
}

// ---------------------------------------------------------------------------
// Generic recurrent step (qwen35.rs:163-225): one thread per (head, value
// column); per column the key loops run in the reference's order.
// ---------------------------------------------------------------------------
__global__ void gdn_step_kernel(float* S, const float* q, const float* k, const float* v,
                                const float* g, const float* beta, uint32_t heads, uint32_t kd,
                                uint32_t vd, float* out) {
  const uint32_t h = blockIdx.y;
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= heads || j >= vd) return;
  float* s = S + uint64_t(h) * kd * vd;
  const float* kk = k + uint64_t(h) * kd;
  const float* qq = q + uint64_t(h) * kd;
  const float decay = expf(g[h]);
  float mem = 0.f;
  for (uint32_t i = 0; i < kd; ++i) {
    const float sv = __fmul_rn(s[uint64_t(i) * vd + j], decay);
    s[uint64_t(i) * vd + j] = sv;
    mem = __fadd_rn(mem, __fmul_rn(sv, kk[i]));
  }
  const float delta = __fmul_rn(__fsub_rn(v[uint64_t(h) * vd + j], mem), beta[h]);
  float r = 0.f;
  for (uint32_t i = 0; i < kd; ++i) {
    const float sv = __fadd_rn(s[uint64_t(i) * vd + j], __fmul_rn(kk[i], delta));
    s[uint64_t(i) * vd + j] = sv;
    r = __fadd_rn(r, __fmul_rn(sv, qq[i]));
  }
  out[uint64_t(h) * vd + j] = r;
}

void launch_gdn_step(float* state, const float* q, const float* k, const float* v,
                     const float* g, const float* beta, uint32_t heads, uint32_t kd,
                     uint32_t vd, float* out, cudaStream_t s) {
  dim3 grid((vd + 127) / 128, heads);
  gdn_step_kernel<<<grid, 128, 0, s>>>(state, q, k, v, g, beta, heads, kd, vd, out);
}

// ---------------------------------------------------------------------------
// Fused Gated DeltaNet layer step (qwen35_runtime.rs:541-620 + qwen35.rs).
// Grid (value heads, kGdnSplit): CTA (h, c) owns value head h and state
// columns [32c, 32c + 32). Its 128 threads each compute the conv + SiLU of one
// q and one k channel of h's key head (every split needs the whole
// normalised q and k), and the first 32 threads the conv of the CTA's 32 v
// channels. For the recurrence, warp w holds rows [32w, 32w + 32) of the
// CTA's 32 columns (lane = column, 32 registers), so a column's two dot
// products (S^T k and S^T q) are four 32-term partial sums added in a fixed
// order across the warps; the per-element updates keep the order of
// qwen35.rs:163-225. Every global load of the step is issued up front after
// the PDL wait, so the step costs about one memory round trip.
// ---------------------------------------------------------------------------
constexpr int kGdnD = 128;
constexpr int kGdnSplit = 4;                 // column splits per value head
constexpr int kGdnCols = kGdnD / kGdnSplit;  // 32 state columns per CTA

template <int K>
__device__ __forceinline__ float conv_silu_fixed(float xin, const float* st, const float* wc) {
  float v = __fmul_rn(xin, wc[K - 1]);
#pragma unroll
  for (int t = 0; t + 1 < K; ++t) v = __fadd_rn(v, __fmul_rn(st[t], wc[t]));
  return v / (1.0f + expf(-v));
}

template <int K>
__global__ void __launch_bounds__(kGdnD) gdn_layer_kernel(const GdnLayerArgs a) {
  __shared__ float qs[kGdnD], ks[kGdnD], vs[kGdnCols];
  __shared__ float red[2][kGdnD / 32];
  __shared__ float part[kGdnD / 32][kGdnCols];
  __shared__ float delta_s[kGdnCols];
  const uint32_t h = blockIdx.x, split = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint32_t kh = a.key_heads, vh = a.value_heads;
  const uint32_t rep = vh / kh, khead = h / rep;
  const uint32_t kw = kh * kGdnD;
  const uint32_t col = split * kGdnCols + lane;  // this thread's state column
  const uint32_t cq = khead * kGdnD + t, ck = kw + cq, cv = 2 * kw + h * kGdnD + col;
  pdl_launch_dependents();
  pdl_wait();
  // the launch's epoch of the peer exchange (the previous grid has finished)
  __shared__ uint32_t s_epoch;
  if (a.xcore.n && t == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(a.xcore.epoch) + 1;
  // ---- every load of the step, independent of one another ----
  float* S = a.state + uint64_t(h) * kGdnD * kGdnD + uint64_t(warp) * kGdnCols * kGdnD + col;
  float s[kGdnCols];
#pragma unroll
  for (int i = 0; i < kGdnCols; ++i) s[i] = S[uint64_t(i) * kGdnD];
  float xin[3], st[3][K - 1], wc[3][K];
  const uint32_t ch[3] = {cq, ck, cv};
  const bool has_v = warp == 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    if (j == 2 && !has_v) {
      xin[j] = 0.f;
#pragma unroll
      for (int u = 0; u + 1 < K; ++u) st[j][u] = 0.f;
#pragma unroll
      for (int u = 0; u < K; ++u) wc[j][u] = 0.f;
      continue;
    }
    xin[j] = a.qkv[ch[j]];
#pragma unroll
    for (int u = 0; u + 1 < K; ++u) st[j][u] = a.conv_in[uint64_t(ch[j]) * (K - 1) + u];
#pragma unroll
    for (int u = 0; u < K; ++u) wc[j][u] = a.conv_w[uint64_t(ch[j]) * K + u];
  }
  float g_in0, g_in1, g_in2, g_in3;
  if (a.gates) {
    g_in0 = a.gates[h];
    g_in1 = a.gates[vh + h];
    g_in2 = g_in3 = 0.f;
  } else if (a.alpha_w) {
    // this head's alpha and beta projections (qwen35_runtime.rs:409-446):
    // rows alpha_w[h], beta_w[h] against x * (1 + norm) * rsqrt(mean x^2 + eps),
    // the RMS factor applied to the two dot products at the end
    const uint32_t cols = a.ab_cols;
    const float* wa = a.alpha_w + uint64_t(h) * cols;
    const float* wb = a.beta_w + uint64_t(h) * cols;
    float ss = 0.f, da = 0.f, db = 0.f;
    if ((cols & 3) == 0 && ((reinterpret_cast<uintptr_t>(wa) | reinterpret_cast<uintptr_t>(wb) |
                             reinterpret_cast<uintptr_t>(a.ab_x) | reinterpret_cast<uintptr_t>(a.ab_norm)) & 15) == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(a.ab_x);
      const float4* n4 = reinterpret_cast<const float4*>(a.ab_norm);
      const float4* a4 = reinterpret_cast<const float4*>(wa);
      const float4* b4 = reinterpret_cast<const float4*>(wb);
      for (uint32_t i = t; i < cols / 4; i += kGdnD) {
        const float4 xv = x4[i], nv = __ldg(n4 + i), av = __ldg(a4 + i), bv = __ldg(b4 + i);
        ss += xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w;
        const float y0 = xv.x * (1.0f + nv.x), y1 = xv.y * (1.0f + nv.y), y2 = xv.z * (1.0f + nv.z),
                    y3 = xv.w * (1.0f + nv.w);
        da += av.x * y0 + av.y * y1 + av.z * y2 + av.w * y3;
        db += bv.x * y0 + bv.y * y1 + bv.z * y2 + bv.w * y3;
      }
    } else {
      for (uint32_t i = t; i < cols; i += kGdnD) {
        const float xv = a.ab_x[i], y = xv * (1.0f + a.ab_norm[i]);
        ss += xv * xv;
        da += wa[i] * y;
        db += wb[i] * y;
      }
    }
    __shared__ float abred[3][kGdnD / 32];
    ss = warp_sum(ss);
    da = warp_sum(da);
    db = warp_sum(db);
    if (lane == 0) {
      abred[0][warp] = ss;
      abred[1][warp] = da;
      abred[2][warp] = db;
    }
    __syncthreads();
    float tss = 0.f, tda = 0.f, tdb = 0.f;
#pragma unroll
    for (int w = 0; w < kGdnD / 32; ++w) {
      tss += abred[0][w];
      tda += abred[1][w];
      tdb += abred[2][w];
    }
    const float inv = 1.0f / sqrtf(tss / float(cols) + a.ab_eps);
    g_in0 = tda * inv;
    g_in1 = a.dt_bias[h];
    g_in2 = a.a_log[h];
    g_in3 = tdb * inv;
  } else {
    g_in0 = a.alpha[h];
    g_in1 = a.dt_bias[h];
    g_in2 = a.a_log[h];
    g_in3 = a.beta_logit[h];
  }
  // ---- conv + SiLU, conv state shift ----
  const float oq = conv_silu_fixed<K>(xin[0], st[0], wc[0]);
  const float ok = conv_silu_fixed<K>(xin[1], st[1], wc[1]);
  if (has_v) vs[lane] = conv_silu_fixed<K>(xin[2], st[2], wc[2]);
  {
    // one CTA per key head owns the q/k conv state; each split its v channels
    const bool write_qk = (h % rep) == 0 && split == 0;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      if (j < 2 && !write_qk) continue;
      if (j == 2 && !has_v) continue;
      float* so = a.conv_out + uint64_t(ch[j]) * (K - 1);
#pragma unroll
      for (int u = 0; u + 2 < K; ++u) so[u] = st[j][u + 1];
      so[K - 2] = xin[j];
    }
  }
  // ---- q/k L2 norms over the key head (CTA reduction) ----
  float sq = warp_sum(oq * oq), sk = warp_sum(ok * ok);
  if (lane == 0) {
    red[0][warp] = sq;
    red[1][warp] = sk;
  }
  __syncthreads();
  sq = (red[0][0] + red[0][1]) + (red[0][2] + red[0][3]);
  sk = (red[1][0] + red[1][1]) + (red[1][2] + red[1][3]);
  const float invq = 1.0f / sqrtf(sq + 1.0e-6f);
  const float invk = 1.0f / sqrtf(sk + 1.0e-6f);
  qs[t] = __fdiv_rn(oq * invq, sqrtf(float(kGdnD)));
  ks[t] = ok * invk;
  // gates (qwen35_runtime.rs:593-601)
  float g, beta;
  if (a.gates) {
    g = g_in0;
    beta = g_in1;
  } else {
    const float sp_in = g_in0 + g_in1;
    const float sp = sp_in > 20.0f ? sp_in : log1pf(expf(sp_in));
    g = -expf(g_in2) * sp;
    beta = 1.0f / (1.0f + expf(-g_in3));
  }
  __syncthreads();
  // ---- recurrence on column `col`, rows [32 warp, 32 warp + 32) ----
  const float decay = expf(g);
  const float* kr = ks + warp * kGdnCols;
  const float* qr = qs + warp * kGdnCols;
  float mem = 0.f;
#pragma unroll
  for (int i = 0; i < kGdnCols; ++i) {
    s[i] = __fmul_rn(s[i], decay);
    mem = __fadd_rn(mem, __fmul_rn(s[i], kr[i]));
  }
  part[warp][lane] = mem;
  __syncthreads();
  if (warp == 0) {
    const float m = __fadd_rn(__fadd_rn(part[0][lane], part[1][lane]), __fadd_rn(part[2][lane], part[3][lane]));
    delta_s[lane] = __fmul_rn(__fsub_rn(vs[lane], m), beta);
  }
  __syncthreads();
  const float delta = delta_s[lane];
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < kGdnCols; ++i) {
    s[i] = __fadd_rn(s[i], __fmul_rn(kr[i], delta));
    r = __fadd_rn(r, __fmul_rn(s[i], qr[i]));
  }
#pragma unroll
  for (int i = 0; i < kGdnCols; ++i) S[uint64_t(i) * kGdnD] = s[i];
  __syncthreads();  // every warp has read part[] for the first reduction
  part[warp][lane] = r;
  __syncthreads();
  if (warp == 0) {
    const float o = __fadd_rn(__fadd_rn(part[0][lane], part[1][lane]), __fadd_rn(part[2][lane], part[3][lane]));
    if (a.xcore.n) {
      // this rank's core and z rows leave for every rank
      const uint32_t row = h * kGdnD + col;
      peer_store_row(a.xcore, s_epoch, row, o);
      peer_store_row(a.xz, s_epoch, row, a.z_in[row]);
    } else {
      a.core[h * kGdnD + col] = o;
    }
  }
  if (a.xcore.n) {
    // this CTA's slices of the gathered core and z, then its ticket
    const uint32_t cta = blockIdx.y * gridDim.x + blockIdx.x, nctas = gridDim.x * gridDim.y;
    peer_unpack(a.xcore, cta, nctas, s_epoch, a.err, t, kGdnD);
    peer_unpack(a.xz, cta, nctas, s_epoch, a.err, t, kGdnD);
    peer_ticket(a.xcore, nctas, s_epoch, t, kGdnD);
  }
}

void launch_gdn_layer(const GdnLayerArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.value_heads, kGdnSplit);
  cfg.blockDim = dim3(kGdnD);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  switch (a.kernel) {
    case 2: cudaLaunchKernelEx(&cfg, gdn_layer_kernel<2>, a); break;
    case 3: cudaLaunchKernelEx(&cfg, gdn_layer_kernel<3>, a); break;
    case 4: cudaLaunchKernelEx(&cfg, gdn_layer_kernel<4>, a); break;
    case 5: cudaLaunchKernelEx(&cfg, gdn_layer_kernel<5>, a); break;
    case 6: cudaLaunchKernelEx(&cfg, gdn_layer_kernel<6>, a); break;
    case 7: cudaLaunchKernelEx(&cfg, gdn_layer_kernel<7>, a); break;
    case 8: cudaLaunchKernelEx(&cfg, gdn_layer_kernel<8>, a); break;
    default: break;  // rejected by the model's config validation
  }
}

// ---------------------------------------------------------------------------
// RoPE (metal.rs:1655-1679) with host-computed inverse frequencies so the
// angle pos*freq is bit-identical to the CPU reference's.
// ---------------------------------------------------------------------------
__global__ void rope_kernel(const float* x, const float* freq, uint32_t heads, uint32_t hd,
                            uint32_t pos, float* out) {
  const uint32_t pairs = hd / 2;
  const uint32_t p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= heads * pairs) return;
  const uint32_t h = p / pairs, i = p % pairs;
  const float ang = float(pos) * freq[i];
  float sn, cs;
  sincosf(ang, &sn, &cs);
  const uint64_t o = uint64_t(h) * hd + 2 * i;
  const float a = x[o], b = x[o + 1];
  out[o] = a * cs - b * sn;
  out[o + 1] = a * sn + b * cs;
}

void launch_rope(const float* x, const float* freq, uint32_t heads, uint32_t hd, uint32_t pos,
                 float* out, cudaStream_t s) {
  const uint32_t n = heads * (hd / 2);
  rope_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, freq, heads, hd, pos, out);
}

// ---------------------------------------------------------------------------
// Split-K GQA decode (metal.rs:1681-1766 semantics) over a head-major cache
// [kvh][cap][hd] (cache.rs:1-4), bf16 or f32 elements, plus the current
// token's K/V in f32. Grid (chunks, kvh), 256 threads. Each CTA handles all
// query heads of its KV group for `chunk` tokens, so K/V are read once.
// ---------------------------------------------------------------------------
constexpr int kAttnThreads = 256;
constexpr int kAttnMaxHd = 256;
constexpr int kAttnMaxGroup = 8;

template <bool BF16>
__device__ __forceinline__ float cache_elem(const void* c, uint64_t i) {
  if (BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(c)[i]);
  return reinterpret_cast<const float*>(c)[i];
}

// q/k preparation: (1+w) head RMSNorm, then RoPE on the first `rotary` dims.
__device__ void prep_head(const float* src, const float* norm_w, const float* freq,
                          uint32_t hd, uint32_t rotary, uint32_t pos, float eps, float* dst,
                          float* red) {
  // one warp per head
  const int lane = threadIdx.x & 31;
  float inv = 1.0f;
  if (norm_w) {
    float ss = 0.f;
    for (uint32_t i = lane; i < hd; i += 32) ss += src[i] * src[i];
    ss = warp_sum(ss);
    inv = 1.0f / sqrtf(ss / float(hd) + eps);
  }
  for (uint32_t i = lane; i < hd; i += 32) dst[i] = norm_w ? src[i] * inv * (1.0f + norm_w[i]) : src[i];
  __syncwarp();
  if (freq) {
    for (uint32_t p = lane; p < rotary / 2; p += 32) {
      const float ang = float(pos) * freq[p];
      float sn, cs;
      sincosf(ang, &sn, &cs);
      const float a = dst[2 * p], b = dst[2 * p + 1];
      dst[2 * p] = a * cs - b * sn;
      dst[2 * p + 1] = a * sn + b * cs;
    }
  }
  __syncwarp();
  (void)red;
}

template <bool BF16>
__global__ void __launch_bounds__(kAttnThreads) attn_partial_kernel(const AttnArgs a) {
  __shared__ float qs[kAttnMaxGroup][kAttnMaxHd];
  __shared__ float kn[kAttnMaxHd];
  __shared__ float sc[kAttnMaxGroup][kAttnThreads];
  __shared__ float red[kAttnMaxGroup][kAttnThreads / 32];
  __shared__ float mx[kAttnMaxGroup], sm[kAttnMaxGroup];
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t kvh = blockIdx.y, chunk = blockIdx.x;
  const uint32_t hd = a.hd, group = a.qh / a.kvh;
  const uint32_t n = a.dev_pos ? a.dev_pos[0] : a.cached;  // cached tokens
  const uint32_t pos = a.dev_pos ? a.dev_pos[0] : a.position;
  const uint32_t total = n + 1;
  const uint32_t t0 = chunk * a.chunk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t nchunks_live = (total + a.chunk - 1) / a.chunk;
  float* part = a.part + (uint64_t(chunk) * a.qh) * (hd + 2);
  if (chunk >= nchunks_live) {
    // beyond the live length (graph launches size the grid for capacity)
    for (uint32_t h = threadIdx.x; h < group; h += blockDim.x) {
      float* ph = part + uint64_t(kvh * group + h) * (hd + 2);
      ph[hd] = -INFINITY;
      ph[hd + 1] = 0.f;
    }
    return;
  }
  const uint32_t cnt = min(a.chunk, total - t0);
  const bool has_new = (t0 + cnt == total);
  // prepare queries of the group (and the new key when this chunk holds it)
  for (uint32_t h = warp; h < group + 1; h += kAttnThreads / 32) {
    if (h < group) {
      const uint32_t qhd = kvh * group + h;
      prep_head(a.q + uint64_t(qhd) * hd, a.q_norm, a.rope_freq, hd, a.rotary, pos, a.eps,
                qs[h], nullptr);
    } else if (has_new || a.k_cache_w) {
      prep_head(a.k_new + uint64_t(kvh) * hd, a.k_norm, a.rope_freq, hd, a.rotary, pos, a.eps,
                kn, nullptr);
    }
  }
  __syncthreads();
  const float scale = 1.0f / sqrtf(float(hd));
  // scores: one thread per token, sequential over dims (reference order)
  for (uint32_t tt = threadIdx.x; tt < cnt; tt += kAttnThreads) {
    const uint32_t t = t0 + tt;
    float acc[kAttnMaxGroup];
#pragma unroll
    for (int h = 0; h < kAttnMaxGroup; ++h) acc[h] = 0.f;
    if (t < n) {
      const uint64_t base = (uint64_t(kvh) * a.cap + t) * hd;
      if (BF16 && (hd % 8 == 0)) {
        const uint4* kr = reinterpret_cast<const uint4*>(
            reinterpret_cast<const __nv_bfloat16*>(a.k_cache) + base);
        for (uint32_t d8 = 0; d8 < hd / 8; ++d8) {
          const uint4 u = __ldg(kr + d8);
          const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float kv = __uint_as_float((wv[e >> 1] >> ((e & 1) * 16)) << 16);
            const uint32_t d = d8 * 8 + e;
#pragma unroll
            for (int h = 0; h < kAttnMaxGroup; ++h)
              if (h < int(group)) acc[h] += qs[h][d] * kv;
          }
        }
      } else {
        for (uint32_t d = 0; d < hd; ++d) {
          const float kv = cache_elem<BF16>(a.k_cache, base + d);
#pragma unroll
          for (int h = 0; h < kAttnMaxGroup; ++h)
            if (h < int(group)) acc[h] += qs[h][d] * kv;
        }
      }
    } else {
      for (uint32_t d = 0; d < hd; ++d) {
        const float kv = kn[d];
#pragma unroll
        for (int h = 0; h < kAttnMaxGroup; ++h)
          if (h < int(group)) acc[h] += qs[h][d] * kv;
      }
    }
#pragma unroll
    for (int h = 0; h < kAttnMaxGroup; ++h)
      if (h < int(group)) sc[h][tt] = acc[h];
  }
  __syncthreads();
  // per-head chunk max of score*scale and sum of exp
  for (uint32_t h = 0; h < group; ++h) {
    float m = -INFINITY;
    for (uint32_t tt = threadIdx.x; tt < cnt; tt += kAttnThreads) m = fmaxf(m, sc[h][tt] * scale);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[h][warp] = m;
  }
  __syncthreads();
  if (threadIdx.x < group) {
    float m = -INFINITY;
    for (int w = 0; w < kAttnThreads / 32; ++w) m = fmaxf(m, red[threadIdx.x][w]);
    mx[threadIdx.x] = m;
  }
  __syncthreads();
  for (uint32_t h = 0; h < group; ++h) {
    float s = 0.f;
    for (uint32_t tt = threadIdx.x; tt < cnt; tt += kAttnThreads) {
      const float p = expf(sc[h][tt] * scale - mx[h]);
      sc[h][tt] = p;
      s += p;
    }
    s = warp_sum(s);
    if (lane == 0) red[h][warp] = s;
  }
  __syncthreads();
  if (threadIdx.x < group) {
    float s = 0.f;
    for (int w = 0; w < kAttnThreads / 32; ++w) s += red[threadIdx.x][w];
    sm[threadIdx.x] = s;
  }
  __syncthreads();
  // P.V: one thread per dimension
  for (uint32_t d = threadIdx.x; d < hd; d += kAttnThreads) {
    float acc[kAttnMaxGroup];
#pragma unroll
    for (int h = 0; h < kAttnMaxGroup; ++h) acc[h] = 0.f;
    for (uint32_t tt = 0; tt < cnt; ++tt) {
      const uint32_t t = t0 + tt;
      const float vv = (t < n) ? cache_elem<BF16>(a.v_cache, (uint64_t(kvh) * a.cap + t) * hd + d)
                               : a.v_new[uint64_t(kvh) * hd + d];
#pragma unroll
      for (int h = 0; h < kAttnMaxGroup; ++h)
        if (h < int(group)) acc[h] += sc[h][tt] * vv;
    }
    for (uint32_t h = 0; h < group; ++h) part[uint64_t(kvh * group + h) * (hd + 2) + d] = acc[h];
  }
  if (threadIdx.x < group) {
    float* ph = part + uint64_t(kvh * group + threadIdx.x) * (hd + 2);
    ph[hd] = mx[threadIdx.x];
    ph[hd + 1] = sm[threadIdx.x];
  }
  // append the new token (bf16) to the cache; position n is never read here
  if (has_new && a.k_cache_w) {
    if (n < a.cap) {
      for (uint32_t d = threadIdx.x; d < hd; d += kAttnThreads) {
        const uint64_t o = (uint64_t(kvh) * a.cap + n) * hd + d;
        a.k_cache_w[o] = __bfloat16_as_ushort(__float2bfloat16_rn(kn[d]));
        a.v_cache_w[o] = __bfloat16_as_ushort(__float2bfloat16_rn(a.v_new[uint64_t(kvh) * hd + d]));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K decode over a bf16 head-major cache on the tensor cores.
//
// Grid (splits, kvh), 128 threads (4 warps), one CTA per SM. Split s of KV
// head h owns the contiguous cached tokens [s*per, (s+1)*per) of that head.
// Tiles of kFaTile tokens of K and V arrive by 3-D TMA (tensor map
// {hd, n, kvh}, box {64, kFaTile, 1}, 128-byte swizzle) in a kFaStages-deep
// shared-memory ring; rows at or beyond the cached length n lie outside the
// map and arrive as zeros. Warp w owns rows 16w..16w+15 of every tile and
// keeps its own online-softmax state (running max, partial sum, f32
// accumulators), so a tile needs one CTA barrier (to recycle the stage):
//   scores  S = Q K^T on mma.m16n8k16 (bf16 in, f32 accumulate). The A rows
//           hold the group's queries split into two bf16 terms, q = hi + lo
//           (rows 0..7 hi, rows 8..15 lo; |q - hi - lo| <= 2^-17 |q|), so the
//           score of head g is C[g] + C[g+8]. K is bf16 already (exact B).
//   softmax running max over the quad of lanes holding head g, rescale
//           factor exp(m_old - m_new), p = exp(s - m_new).
//   P.V     the score fragments ARE the A fragments of the next MMA: p is
//           split hi/lo into rows g / g+8 again and multiplied by V through
//           ldmatrix.trans, accumulating all head dims in registers.
// The last split also scores the current token (f32 K/V) and appends it to
// the cache as bf16. Warps merge through shared memory into the CTA's
// partial (acc, m, l) per query head in part[split][qh][hd+2];
// attn_merge_kernel combines the splits.
// ---------------------------------------------------------------------------
constexpr int kFaThreads = 128;
constexpr int kFaWarps = kFaThreads / 32;
constexpr int kFaTile = 16 * kFaWarps;  // tokens per staged tile (16 per warp)
constexpr int kFaStages = 3;
constexpr int kFaCtas = 148;            // one CTA per SM on B200
constexpr uint32_t kFaBox = uint32_t(kFaTile) * 128u;  // one TMA box: kFaTile rows x 128 bytes

__device__ __forceinline__ uint64_t umin64(uint64_t a, uint64_t b) { return a < b ? a : b; }

// bf16 pair (lo element first) of round-to-nearest-even conversions.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  return uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(lo))) |
         (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(hi))) << 16);
}
// x = hi + lo in bf16: returns the hi pair and writes the lo pair.
__device__ __forceinline__ uint32_t split_bf16x2(float x0, float x1, uint32_t& lo) {
  const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
  lo = pack_bf16(x0 - __bfloat162float(h0), x1 - __bfloat162float(h1));
  return uint32_t(__bfloat16_as_ushort(h0)) | (uint32_t(__bfloat16_as_ushort(h1)) << 16);
}

__device__ __forceinline__ void mma_bf16_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// 3-D tiled TMA load (no multicast; the source is this GPU's cache).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

template <int HD, int G>
struct FaLayout {
  static constexpr uint32_t nbox = HD / 64;                     // boxes per K (or V) tile
  static constexpr uint32_t stage_bytes = 2u * nbox * kFaBox;    // K boxes then V boxes
  static constexpr uint32_t pitch = HD + 8;                      // bf16 per row of the query A matrix
  static constexpr uint32_t qa_off = kFaStages * stage_bytes;    // bf16 [16][pitch]
  static constexpr uint32_t qs_off = qa_off + 16 * pitch * 2;    // float [G][HD]
  static constexpr uint32_t kn_off = qs_off + G * HD * 4;        // float [HD]
  static constexpr uint32_t mw_off = kn_off + HD * 4;            // float m[warps][8], l[warps][8], wt[warps][8]
  static constexpr uint32_t bar_off = (mw_off + 3 * kFaWarps * 8 * 4 + 15) & ~15u;  // u64 full[kFaStages]
  static constexpr uint32_t bytes = bar_off + kFaStages * 8 + 1024;  // + alignment slack
  static_assert(kFaWarps * G * HD * 4 <= kFaStages * stage_bytes, "warp merge aliases the ring");
};

template <int HD, int G>
__global__ void __launch_bounds__(kFaThreads, 1)
    attn_split_bf16_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                           const AttnArgs a, uint32_t nsplit) {
  using L = FaLayout<HD, G>;
  constexpr int KS = HD / 16;  // k-steps of the score MMA
  constexpr int NB = HD / 8;   // 8-dim n-blocks of the P.V MMA
  extern __shared__ __align__(1024) uint8_t fsm_raw[];
  // 128-byte swizzled TMA destinations need 1024-byte alignment
  uint8_t* fsm = fsm_raw + ((1024u - (smem_u32(fsm_raw) & 1023u)) & 1023u);
  const uint32_t ring = smem_u32(fsm);
  uint16_t* qa = reinterpret_cast<uint16_t*>(fsm + L::qa_off);
  float* qs = reinterpret_cast<float*>(fsm + L::qs_off);
  float* kn = reinterpret_cast<float*>(fsm + L::kn_off);
  float* mw = reinterpret_cast<float*>(fsm + L::mw_off);  // [warps][8]
  float* lw = mw + kFaWarps * 8;
  float* wt = lw + kFaWarps * 8;
  uint64_t* full = reinterpret_cast<uint64_t*>(fsm + L::bar_off);
  float* scratch = reinterpret_cast<float*>(fsm);  // ring, reused after the last tile

  pdl_launch_dependents();
  pdl_wait();
  const uint32_t hkv = blockIdx.y, split = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;  // MMA fragment row / column pair
  const uint32_t n = a.cached;
  const uint32_t per = uint32_t((uint64_t(n) + nsplit - 1) / nsplit);
  const uint32_t tb = uint32_t(umin64(n, uint64_t(split) * per));
  const uint32_t te = uint32_t(umin64(n, uint64_t(tb) + per));
  const bool last = split + 1 == nsplit;
  const uint32_t ntile = (te - tb + kFaTile - 1) / kFaTile;
  float* parts = a.part;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFaStages; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  const uint64_t pol = l2_policy_evict_first();
  auto issue = [&](uint32_t i) {
    const int t0 = int(tb + i * kFaTile);
    const uint32_t st = ring + (i % kFaStages) * L::stage_bytes;
    uint64_t* bar = &full[i % kFaStages];
    mbar_arrive_expect_tx(bar, L::stage_bytes);
#pragma unroll
    for (uint32_t j = 0; j < L::nbox; ++j) {
      tma_load_3d(st + j * kFaBox, &tk, int(j * 64), t0, int(hkv), bar, pol);
      tma_load_3d(st + (L::nbox + j) * kFaBox, &tv, int(j * 64), t0, int(hkv), bar, pol);
    }
  };
  if (threadIdx.x == 0)
    for (uint32_t i = 0; i < ntile && i < kFaStages; ++i) issue(i);

  // queries of the group (and the current key when this split holds it)
  for (int h = warp; h < G + 1; h += kFaWarps) {
    if (h < G)
      prep_head(a.q + uint64_t(hkv * G + h) * HD, a.q_norm, a.rope_freq, HD, a.rotary, a.position, a.eps,
                qs + h * HD, nullptr);
    else if (last)
      prep_head(a.k_new + uint64_t(hkv) * HD, a.k_norm, a.rope_freq, HD, a.rotary, a.position, a.eps, kn,
                nullptr);
  }
  __syncthreads();
  // query A matrix: row h = hi(q_h), row 8+h = lo(q_h); rows of absent heads are 0
  for (int idx = threadIdx.x; idx < 8 * HD; idx += kFaThreads) {
    const int h = idx / HD, d = idx % HD;
    const float x = h < G ? qs[h * HD + d] : 0.f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(x);
    qa[h * L::pitch + d] = __bfloat16_as_ushort(hi);
    qa[(8 + h) * L::pitch + d] = __bfloat16_as_ushort(__float2bfloat16_rn(x - __bfloat162float(hi)));
  }
  __syncthreads();
  const uint32_t qa_lane = smem_u32(qa) + (((lane & 7) + ((lane >> 3) & 1) * 8) * L::pitch + (lane >> 4) * 8) * 2;

  float m_run = -INFINITY, l_run = 0.f;
  float acc[NB][4];
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[b][e] = 0.f;
  const float scale = 1.0f / sqrtf(float(HD));
  bool bad = false;

  for (uint32_t i = 0; i < ntile; ++i) {
    const uint32_t stg = i % kFaStages;
    const bool ok = mbar_wait_bounded(&full[stg], (i / kFaStages) & 1);
    if (__syncthreads_or(!ok)) {
      // give up: record it, wait (bounded) for this CTA's copies in flight
      if (threadIdx.x == 0) {
        if (a.err) atomicOr(a.err, KERR_TIMEOUT_FULL);
        for (uint32_t j = i; j < ntile && j < i + kFaStages; ++j)
          if (!mbar_wait_bounded(&full[j % kFaStages], (j / kFaStages) & 1) && a.err)
            atomicOr(a.err, KERR_TIMEOUT_DRAIN);
      }
      bad = true;
      break;
    }
    const uint32_t kt = ring + stg * L::stage_bytes;
    const uint32_t vt = kt + L::nbox * kFaBox;
    const int r0 = warp * 16;
    const int valid = int(te - (tb + i * kFaTile)) - r0;  // rows of this warp that are live
    if (valid > 0) {
      // scores of rows r0..r0+15: two n-blocks, even/odd k-steps on separate accumulators
      float sc[2][2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[j][p][e] = 0.f;
#pragma unroll
      for (int s = 0; s < KS; s += 2) {
        uint32_t aA[4], aB[4];
        ldsm_x4(qa_lane + s * 32, aA);
        ldsm_x4(qa_lane + (s + 1) * 32, aB);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t b[4];
          ldsm_x4(kt + (s >> 2) * kFaBox + swz(r0 + j * 8 + (lane & 7), (s & 3) * 2 + (lane >> 3)), b);
          mma_bf16_16816(sc[j][0], aA, b[0], b[1]);
          mma_bf16_16816(sc[j][1], aB, b[2], b[3]);
        }
      }
      float sv[2][2];
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = ((sc[j][0][e] + sc[j][0][e + 2]) + (sc[j][1][e] + sc[j][1][e + 2])) * scale;
          sv[j][e] = (j * 8 + 2 * c + e) < valid ? v : -INFINITY;
          mt = fmaxf(mt, sv[j][e]);
        }
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      const float mn = fmaxf(m_run, mt);
      const float al = expf(m_run - mn);
      float pv[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) pv[j][e] = expf(sv[j][e] - mn);
      l_run = l_run * al + ((pv[0][0] + pv[0][1]) + (pv[1][0] + pv[1][1]));
      m_run = mn;
      uint32_t ap[4];
      ap[0] = split_bf16x2(pv[0][0], pv[0][1], ap[1]);
      ap[2] = split_bf16x2(pv[1][0], pv[1][1], ap[3]);
      const uint32_t vrow = r0 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
      for (int pb = 0; pb < NB / 2; ++pb) {
        const uint32_t dchunk = pb * 2 + (lane >> 4);  // 8-dim chunk of the head
        uint32_t b[4];
        ldsm_x4_trans(vt + (dchunk >> 3) * kFaBox + swz(vrow, dchunk & 7), b);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[2 * pb][e] *= al;
          acc[2 * pb + 1][e] *= al;
        }
        mma_bf16_16816(acc[2 * pb], ap, b[0], b[1]);
        mma_bf16_16816(acc[2 * pb + 1], ap, b[2], b[3]);
      }
    }
    __syncthreads();  // stage free
    if (threadIdx.x == 0 && i + kFaStages < ntile) issue(i + kFaStages);
  }
  if (bad) {
    m_run = -INFINITY;
    l_run = 0.f;
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[b][e] = 0.f;
  }

  if (last && !bad && warp == 0) {
    // the current token: score from the prepared key, value from v_new
    float sn = -INFINITY;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float d = 0.f;
      for (int j = lane; j < HD; j += 32) d += qs[h * HD + j] * kn[j];
      d = warp_sum(d) * scale;
      if (g == h) sn = d;
    }
    if (g < G) {
      const float mn = fmaxf(m_run, sn);
      const float al = expf(m_run - mn), p = expf(sn - mn);
      l_run = l_run * al + (c == 0 ? p : 0.f);
      m_run = mn;
      const float* vn = a.v_new + uint64_t(hkv) * HD + 2 * c;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        acc[b][0] = fmaf(p, vn[b * 8], acc[b][0] * al);
        acc[b][1] = fmaf(p, vn[b * 8 + 1], acc[b][1] * al);
        acc[b][2] *= al;
        acc[b][3] *= al;
      }
    }
  }
  if (last && a.k_cache_w && n < a.cap) {
    for (int d = threadIdx.x; d < HD; d += kFaThreads) {
      const uint64_t o = (uint64_t(hkv) * a.cap + n) * HD + d;
      a.k_cache_w[o] = __bfloat16_as_ushort(__float2bfloat16_rn(kn[d]));
      a.v_cache_w[o] = __bfloat16_as_ushort(__float2bfloat16_rn(a.v_new[uint64_t(hkv) * HD + d]));
    }
  }

  // ---- merge the warps: partial (acc, m, l) of this split ------------------
  float lq = l_run + __shfl_xor_sync(0xffffffffu, l_run, 1);
  lq += __shfl_xor_sync(0xffffffffu, lq, 2);
  __syncthreads();  // ring no longer read
  if (g < G) {
    if (c == 0) {
      mw[warp * 8 + g] = m_run;
      lw[warp * 8 + g] = lq;
    }
    float* dst = scratch + (warp * G + g) * HD + 2 * c;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      dst[b * 8] = acc[b][0] + acc[b][2];
      dst[b * 8 + 1] = acc[b][1] + acc[b][3];
    }
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float M = -INFINITY;
    for (int w = 0; w < kFaWarps; ++w) M = fmaxf(M, mw[w * 8 + h]);
    float l = 0.f;
    for (int w = 0; w < kFaWarps; ++w) {
      const float x = mw[w * 8 + h] > -INFINITY ? expf(mw[w * 8 + h] - M) : 0.f;
      wt[w * 8 + h] = x;
      l += x * lw[w * 8 + h];
    }
    float* ph = parts + (uint64_t(split) * a.qh + hkv * G + h) * (HD + 2);
    ph[HD] = M;
    ph[HD + 1] = l;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * HD; idx += kFaThreads) {
    const int h = idx / HD, d = idx % HD;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kFaWarps; ++w) s = fmaf(wt[w * 8 + h], scratch[(w * G + h) * HD + d], s);
    parts[(uint64_t(split) * a.qh + hkv * G + h) * (HD + 2) + d] = s;
  }

}

// Merge split partials: out = sum_s w_s acc_s / sum_s w_s l_s with
// w_s = exp(m_s - max m). Grid (qh, hd/32), 256 threads: lane = head dim,
// warp w takes splits w, w+8, ...; a batch of kMergeBatch splits is loaded
// into registers before the split maxima are known, so a merge of up to
// kMergeBatch splits costs one round trip to L2. Fixed summation order.
constexpr int kMergeDims = 32;
constexpr int kMergeWarps = 8;
constexpr int kMergePerLane = 19;
constexpr uint32_t kMergeBatch = kMergeWarps * kMergePerLane;  // 152 splits
constexpr uint32_t kMergeMaxSplits = 4096;

__global__ void __launch_bounds__(kMergeDims * kMergeWarps)
    attn_merge_kernel(const __grid_constant__ AttnArgs a, uint32_t nsplit) {
  __shared__ float sw[kMergeMaxSplits];
  __shared__ float red[kMergeWarps][kMergeDims + 1];
  __shared__ float rm[kMergeWarps], rl[kMergeWarps];
  __shared__ uint32_t s_epoch;
  pdl_launch_dependents();
  pdl_wait();
  // the launch's epoch of the peer exchange (the previous grid has finished)
  if (a.xatt.n && threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(a.xatt.epoch) + 1;
  const uint32_t qhd = blockIdx.x, hd = a.hd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t d = blockIdx.y * kMergeDims + lane;
  const bool live = d < hd;
  const uint64_t stride = uint64_t(a.qh) * (hd + 2);
  const float* base = a.part + uint64_t(qhd) * (hd + 2);
  // first batch of partial values, independent of the weights
  float x[kMergePerLane];
#pragma unroll
  for (int i = 0; i < kMergePerLane; ++i) {
    const uint32_t s = warp + kMergeWarps * i;
    x[i] = (live && s < nsplit) ? __ldcg(base + s * stride + d) : 0.f;
  }
  // split maxima and weights
  float M = -INFINITY;
  for (uint32_t s = threadIdx.x; s < nsplit; s += blockDim.x) {
    const float m = __ldcg(base + s * stride + hd);
    sw[s] = m;
    M = fmaxf(M, m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  if (lane == 0) rm[warp] = M;
  __syncthreads();
  M = rm[0];
#pragma unroll
  for (int w = 1; w < kMergeWarps; ++w) M = fmaxf(M, rm[w]);
  float l = 0.f;
  for (uint32_t s = threadIdx.x; s < nsplit; s += blockDim.x) {
    const float m = sw[s];
    const float w = m > -INFINITY ? expf(m - M) : 0.f;
    sw[s] = w;
    l += w * __ldcg(base + s * stride + hd + 1);
  }
  l = warp_sum(l);
  if (lane == 0) rl[warp] = l;
  __syncthreads();
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < kMergePerLane; ++i) {
    const uint32_t s = warp + kMergeWarps * i;
    if (s < nsplit) acc = fmaf(sw[s], x[i], acc);
  }
  for (uint32_t b0 = kMergeBatch; b0 < nsplit; b0 += kMergeBatch) {  // long generic-kernel caches
#pragma unroll
    for (int i = 0; i < kMergePerLane; ++i) {
      const uint32_t s = b0 + warp + kMergeWarps * i;
      x[i] = (live && s < nsplit) ? __ldcg(base + s * stride + d) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kMergePerLane; ++i) {
      const uint32_t s = b0 + warp + kMergeWarps * i;
      if (s < nsplit) acc = fmaf(sw[s], x[i], acc);
    }
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0) {
    float L = 0.f, o = 0.f;
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) {
      L += rl[w];
      o += red[w][lane];
    }
    if (live) {
      const uint32_t row = qhd * hd + d;
      if (a.xatt.n) {
        // this rank's output and gate rows leave for every rank
        peer_store_row(a.xatt, s_epoch, row, o / L);
        peer_store_row(a.xgate, s_epoch, row, a.gate_in[row]);
      } else {
        a.out[uint64_t(qhd) * hd + d] = o / L;
      }
    }
  }
  if (a.xatt.n) {
    // this CTA's slices of the gathered output and gate, then its ticket
    const uint32_t cta = blockIdx.y * gridDim.x + blockIdx.x, nctas = gridDim.x * gridDim.y;
    peer_unpack(a.xatt, cta, nctas, s_epoch, a.err, threadIdx.x, blockDim.x);
    peer_unpack(a.xgate, cta, nctas, s_epoch, a.err, threadIdx.x, blockDim.x);
    peer_ticket(a.xatt, nctas, s_epoch, threadIdx.x, blockDim.x);
  }
}

// Splits the tensor-core split kernel uses for `n` cached tokens over `kvh` heads:
// at least one tile per split, one CTA per SM in total.
static uint32_t fa_splits(uint32_t kvh, uint32_t n) {
  const uint32_t by_len = (n + kFaTile - 1) / kFaTile;
  const uint32_t by_sm = kvh >= kFaCtas ? 1u : kFaCtas / kvh;
  return max(1u, min(by_len, by_sm));
}

uint64_t attn_scratch_floats(uint32_t qh, uint32_t kvh, uint32_t hd, uint32_t total_tokens, uint32_t chunk) {
  const uint64_t generic = (uint64_t(total_tokens) + chunk - 1) / chunk;
  const uint64_t fast = fa_splits(kvh ? kvh : 1, total_tokens);
  return std::max(generic, fast) * qh * (hd + 2);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// Tensor map over a head-major bf16 cache [kvh][cap][hd] clipped to the first
// n tokens of every head (rows >= n read as zeros), box {64, kFaTile, 1}.
static bool cache_tensor_map(CUtensorMap* map, const void* base, uint32_t hd, uint32_t n, uint32_t kvh,
                             uint32_t cap) {
  auto enc = tensor_map_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  const cuuint64_t dims[3] = {hd, n ? n : 1u, kvh};
  const cuuint64_t strides[2] = {cuuint64_t(hd) * 2, cuuint64_t(cap) * hd * 2};
  const cuuint32_t box[3] = {64, uint32_t(kFaTile), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HD, int G>
static void launch_fa(const CUtensorMap& tk, const CUtensorMap& tv, const AttnArgs& a, cudaLaunchConfig_t cfg,
                      uint32_t nsplit) {
  static std::atomic<uint32_t> smem_limit[kMaxDevices];  // per instantiation and device
  constexpr uint32_t smem = FaLayout<HD, G>::bytes;
  raise_smem_limit(attn_split_bf16_kernel<HD, G>, smem, smem_limit);  // a failure shows in the launch
  cfg.gridDim = dim3(nsplit, a.kvh);
  cfg.blockDim = dim3(kFaThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchKernelEx(&cfg, attn_split_bf16_kernel<HD, G>, tk, tv, a, nsplit);
}

template <int HD>
static bool launch_fa_hd(const AttnArgs& a, const cudaLaunchConfig_t& cfg, uint32_t nsplit, uint32_t g) {
  CUtensorMap tk, tv;
  if (!cache_tensor_map(&tk, a.k_cache, HD, a.cached, a.kvh, a.cap) ||
      !cache_tensor_map(&tv, a.v_cache, HD, a.cached, a.kvh, a.cap))
    return false;
  switch (g) {
    case 1: launch_fa<HD, 1>(tk, tv, a, cfg, nsplit); return true;
    case 2: launch_fa<HD, 2>(tk, tv, a, cfg, nsplit); return true;
    case 3: launch_fa<HD, 3>(tk, tv, a, cfg, nsplit); return true;
    case 4: launch_fa<HD, 4>(tk, tv, a, cfg, nsplit); return true;
    case 5: launch_fa<HD, 5>(tk, tv, a, cfg, nsplit); return true;
    case 6: launch_fa<HD, 6>(tk, tv, a, cfg, nsplit); return true;
    case 7: launch_fa<HD, 7>(tk, tv, a, cfg, nsplit); return true;
    case 8: launch_fa<HD, 8>(tk, tv, a, cfg, nsplit); return true;
  }
  return false;
}

void launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const uint32_t g = a.qh / a.kvh;
  uint32_t nsplit = 0;
  // the tensor-core split kernel: bf16 cache, hd 128 or 256, group <= 8,
  // host-known length
  if (a.cache_bf16 && !a.dev_pos && g >= 1 && g <= 8 && (a.hd == 128 || a.hd == 256)) {
    // programmatic launch: the kernel waits for its predecessor before it
    // reads or writes anything
    cfg.numAttrs = 1;
    nsplit = fa_splits(a.kvh, a.cached);
    if (!(a.hd == 256 ? launch_fa_hd<256>(a, cfg, nsplit, g) : launch_fa_hd<128>(a, cfg, nsplit, g))) nsplit = 0;
  }
  if (!nsplit) {
    // generic kernel: any head size <= 256, f32 or bf16 cache
    const uint32_t max_total = a.dev_pos ? a.cap + 1 : a.cached + 1;
    nsplit = (max_total + a.chunk - 1) / a.chunk;
    cfg.gridDim = dim3(nsplit, a.kvh);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = 0;
    if (a.cache_bf16)
      cudaLaunchKernelEx(&cfg, attn_partial_kernel<true>, a);
    else
      cudaLaunchKernelEx(&cfg, attn_partial_kernel<false>, a);
  }
  // the merge always overlaps its launch with the split kernel's tail
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(a.qh, (a.hd + kMergeDims - 1) / kMergeDims);
  cfg.blockDim = dim3(kMergeDims * kMergeWarps);
  cfg.dynamicSmemBytes = 0;
  cudaLaunchKernelEx(&cfg, attn_merge_kernel, a, nsplit);
}

// ---------------------------------------------------------------------------
// All-gather over NVLink peer memory (one CTA per destination rank).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) p2p_allgather_kernel(const P2PGather g) {
  const uint32_t p = blockIdx.x;  // destination rank
  uint8_t* dst_block = g.block[p];
#pragma unroll
  for (int v = 0; v < 2; ++v) {
    const uint32_t cnt = g.count[v];
    if (cnt == 0) continue;
    const float* src = g.send[v];
    float* dst = reinterpret_cast<float*>(dst_block + g.recv_off[v]) + uint64_t(g.rank) * cnt;
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
      const uint32_t c4 = cnt / 4;
      for (uint32_t i = threadIdx.x; i < c4; i += blockDim.x)
        reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
      for (uint32_t i = c4 * 4 + threadIdx.x; i < cnt; i += blockDim.x) dst[i] = src[i];
    } else {
      for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) dst[i] = src[i];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // every thread's stores above are ordered (bar.sync, then this cumulative
    // system-scope fence) before the flag
    uint32_t* flag = reinterpret_cast<uint32_t*>(dst_block + g.flag_off + 64ull * g.rank);
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(g.epoch) : "memory");
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const long long t0 = clock64(), bound = g.wait_cycles > 0 ? g.wait_cycles : kWaitCycles;
    for (uint32_t q = 0; q < g.n; ++q) {
      if (q == g.rank) continue;
      const uint32_t* f = reinterpret_cast<const uint32_t*>(g.block[g.rank] + g.flag_off + 64ull * q);
      while (true) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if (int32_t(v - g.epoch) >= 0) break;
        if (clock64() - t0 > bound) {
          if (g.err) atomicOr(g.err, KERR_TIMEOUT_FULL);
          return;
        }
      }
    }
  }
}

void launch_p2p_allgather(const P2PGather& g, cudaStream_t s) {
  p2p_allgather_kernel<<<g.n, 256, 0, s>>>(g);
}

// ---------------------------------------------------------------------------
// Greedy argmax under f32::total_cmp, last index among equal maxima.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long argmax_key(float f, uint32_t idx) {
  const int32_t i = __float_as_int(f);
  const int32_t t = i ^ int32_t(uint32_t(i >> 31) >> 1);
  const uint32_t u = uint32_t(t) ^ 0x80000000u;
  return (static_cast<unsigned long long>(u) << 32) | idx;
}

__global__ void argmax_kernel(const float* v, uint64_t n, uint32_t base, unsigned long long* key) {
  unsigned long long best = 0;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const float f = v[i];
    if (isfinite(f)) {
      const unsigned long long k = argmax_key(f, uint32_t(i) + base);
      best = k > best ? k : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0 && best) atomicMax(key, best);
}

// Max over `count` keys (one per rank) -> index; 0xFFFFFFFF when none finite.
__global__ void argmax_finish(unsigned long long* keys, uint32_t count, uint32_t* index) {
  unsigned long long k = 0;
  for (uint32_t i = 0; i < count; ++i) k = keys[i] > k ? keys[i] : k;
  *index = k ? uint32_t(k & 0xffffffffu) : 0xffffffffu;
}

void launch_argmax_key(const float* v, uint64_t n, uint32_t base, unsigned long long* key,
                       cudaStream_t s) {
  uint64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks == 0) blocks = 1;
  argmax_kernel<<<unsigned(blocks), 256, 0, s>>>(v, n, base, key);
}

void launch_argmax_finish(unsigned long long* keys, uint32_t count, uint32_t* index,
                          cudaStream_t s) {
  argmax_finish<<<1, 1, 0, s>>>(keys, count, index);
}

void launch_argmax(const float* v, uint64_t n, unsigned long long* key, uint32_t* index,
                   cudaStream_t s) {
  cudaMemsetAsync(key, 0, sizeof(unsigned long long), s);
  launch_argmax_key(v, n, 0, key, s);
  launch_argmax_finish(key, 1, index, s);
}

// ---------------------------------------------------------------------------
// F32 matvec with the (1+w) RMSNorm of x fused in (alpha/beta projections of
// the Gated DeltaNet mixer, qwen35_runtime.rs:575-590). One CTA per 8 rows.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) f32_matvec_norm_kernel(const float* w0, float* y0, const float* w1,
                                                              float* y1, uint32_t cols, const float* x,
                                                              const float* nw, float eps) {
  // one CTA per output row: the row's loads are all in flight at once
  __shared__ float red[32];
  const bool second = blockIdx.y == 1;
  const float* wr = (second ? w1 : w0) + uint64_t(blockIdx.x) * cols;
  pdl_launch_dependents();
  float acc = 0.f, ss = 0.f;
  if ((cols & 3) == 0 && ((reinterpret_cast<uintptr_t>(wr) | reinterpret_cast<uintptr_t>(x) |
                           reinterpret_cast<uintptr_t>(nw)) & 15) == 0) {
    const float4* w4 = reinterpret_cast<const float4*>(wr);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const float4* n4 = reinterpret_cast<const float4*>(nw);
    pdl_wait();
    for (uint32_t i = threadIdx.x; i < cols / 4; i += blockDim.x) {
      const float4 wv = __ldg(w4 + i), xv = x4[i], nv = __ldg(n4 + i);
      ss += xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w;
      acc += wv.x * (xv.x * (1.0f + nv.x)) + wv.y * (xv.y * (1.0f + nv.y)) + wv.z * (xv.z * (1.0f + nv.z)) +
             wv.w * (xv.w * (1.0f + nv.w));
    }
  } else {
    pdl_wait();
    for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
      ss += x[i] * x[i];
      acc += wr[i] * (x[i] * (1.0f + nw[i]));
    }
  }
  // (1+w) RMSNorm of x is a common factor: sum w*x*(1+nw) * inv
  const float tot = block_sum(ss, red);
  __syncthreads();
  const float dot = block_sum(acc, red);
  const float inv = 1.0f / sqrtf(tot / float(cols) + eps);
  if (threadIdx.x == 0) (second ? y1 : y0)[blockIdx.x] = dot * inv;
}

void launch_f32_matvec_norm2(const float* w0, float* y0, const float* w1, float* y1, uint32_t rows, uint32_t cols,
                             const float* x, const float* norm_w, float eps, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows, w1 ? 2 : 1);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, f32_matvec_norm_kernel, w0, y0, w1, y1, cols, x, norm_w, eps);
}

// ---------------------------------------------------------------------------
// Embedding row (qwen35_runtime.rs:2122-2130): the Q4_K row of the token held
// on this rank (table rows [row_lo, row_hi)) is staged through shared memory
// and dequantized bit-exactly; other ranks write zeros (summed afterwards).
// `table` may be mapped host memory (zero-copy read of one row).
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const uint8_t* table, uint32_t cols, const uint32_t* d_token,
                             uint32_t row_lo, uint32_t row_hi, float* out) {
  extern __shared__ __align__(16) uint8_t row[];
  const uint32_t tok = *d_token;
  const bool mine = tok >= row_lo && tok < row_hi;
  const uint32_t rb = cols / 256 * 144;
  if (mine) {
    const uint4* src = reinterpret_cast<const uint4*>(table + uint64_t(tok - row_lo) * rb);
    for (uint32_t i = threadIdx.x; i < rb / 16; i += blockDim.x) reinterpret_cast<uint4*>(row)[i] = src[i];
  }
  __syncthreads();
  for (uint32_t e = threadIdx.x; e < cols; e += blockDim.x)
    out[e] = mine ? deq_elem(SI_GGML_TYPE_Q4_K, row + (e >> 8) * 144, int(e & 255)) : 0.0f;
}

void launch_embed(const uint8_t* table, uint32_t cols, const uint32_t* d_token, uint32_t row_lo,
                  uint32_t row_hi, float* out, cudaStream_t s) {
  embed_kernel<<<1, 1024, cols / 256 * 144, s>>>(table, cols, d_token, row_lo, row_hi, out);
}

__global__ void add_kernel(const float* a, const float* b, float* y, uint64_t n) {
  const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = a[i] + b[i];
}

void launch_add(const float* a, const float* b, float* y, uint64_t n, cudaStream_t s) {
  add_kernel<<<unsigned((n + 255) / 256), 256, 0, s>>>(a, b, y, n);
}

// SwiGLU of separately computed gate and up rows: y = silu(g) * u, the
// formula of the fused pair epilogue.
__global__ void swiglu_kernel(const float* g, const float* u, float* y, uint64_t n) {
  const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

void launch_swiglu(const float* g, const float* u, float* y, uint64_t n, cudaStream_t s) {
  swiglu_kernel<<<unsigned((n + 255) / 256), 256, 0, s>>>(g, u, y, n);
}

// Gated attention output of `batch` candidates (qwen35_runtime.rs:1206-1214):
// out[k][i] = a[k][i] / (1 + exp(-gate[k][i])).
__global__ void siggate_many_kernel(const float* a, uint64_t lda, const float* gate, uint64_t ldg, float* out,
                                    uint64_t ldo, uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x, k = blockIdx.y;
  if (i < n) out[k * ldo + i] = a[k * lda + i] / (1.0f + expf(-gate[k * ldg + i]));
}

void launch_siggate_many(const float* a, uint64_t lda, const float* gate, uint64_t ldg, float* out, uint64_t ldo,
                         uint32_t n, uint32_t batch, cudaStream_t s) {
  siggate_many_kernel<<<dim3((n + 255) / 256, batch), 256, 0, s>>>(a, lda, gate, ldg, out, ldo, n);
}

}  // namespace si
