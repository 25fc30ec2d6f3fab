// Launchers for the non-matvec kernels of the decode path.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "qmatvec.cuh"  // PeerOut

namespace si {

// Bit-exact dequantization of `elements` values (quant.rs:18-174).
void launch_dequant(uint32_t type, const uint8_t* w, uint64_t elements, float* out,
                    cudaStream_t s);
// F32 row-major matvec (metal.rs:263-305); rows x cols, cols % 4 == 0.
void launch_f32_matvec(const float* w, uint64_t rows, uint64_t cols, const float* x, float* y,
                       cudaStream_t s);
// Head RMSNorm with (1 + w) (qwen35.rs:53-86) and gated RMSNorm (qwen35.rs:14-49).
void launch_rms_norm_heads(const float* x, const float* w, uint32_t heads, uint32_t hd,
                           float eps, float* out, cudaStream_t s);
void launch_rms_norm_gated(const float* x, const float* z, const float* w, uint32_t heads,
                           uint32_t hd, float eps, float* out, cudaStream_t s);
// Causal depthwise conv step (qwen35.rs:93-130): state_in -> state_out.
void launch_conv1d_step(const float* x, const float* state_in, const float* w,
                        uint32_t channels, uint32_t kernel, float* out, float* state_out,
                        cudaStream_t s);
// Generic recurrent step (qwen35.rs:163-225), state updated in place.
void launch_gdn_step(float* state, const float* q, const float* k, const float* v,
                     const float* g, const float* beta, uint32_t heads, uint32_t kd,
                     uint32_t vd, float* out, cudaStream_t s);

// Fused Gated DeltaNet token step of one layer (conv + L2 norm + head repeat +
// gates + recurrence). Core output [value_heads * 128]; the gated RMSNorm is
// applied by the ssm_out matvec prologue.
struct GdnLayerArgs {
  const float* qkv;        // projection output [2*kh*128 + vh*128]
  const float* conv_w;     // [channels][kernel]
  const float* conv_in;    // conv state read  [channels][kernel-1]
  float* conv_out;         // conv state write (the other ping-pong buffer)
  float* state;            // recurrent state [vh][128][128]
  const float* gates;      // if non-null: [g[vh], beta[vh]] supplied directly
  const float* alpha;      // else: alpha/beta projection outputs [vh] each
  const float* beta_logit;
  // else, with alpha_w set, the projections are made here: alpha_w / beta_w
  // F32 rows [vh][ab_cols] over the (1+w) RMSNorm (ab_norm, ab_eps) of ab_x
  const float* alpha_w;
  const float* beta_w;
  const float* ab_x;
  const float* ab_norm;
  uint32_t ab_cols;
  float ab_eps;
  const float* a_log;
  const float* dt_bias;
  float* core;             // [vh*128]
  uint32_t key_heads, value_heads, kernel;
  // row-sharded model (xcore.n > 0): this rank's core rows and its z rows
  // (z_in, [vh*128], the z projection's output) are gathered inside this
  // kernel into every rank's full core and z vectors (xcore.y, xz.y), with
  // the in-kernel exchange of the tensor-core matvecs (peer_exchange.cuh;
  // the two share the ticket and the epoch)
  PeerOut xcore, xz;
  const float* z_in;
  int* err;                // device error word for a timed-out exchange (may be null)
};
void launch_gdn_layer(const GdnLayerArgs& a, cudaStream_t s, bool pdl);

// Attention: rope table, fused q/k norm + partial RoPE + split-K decode over a
// head-major cache, and the combine of the chunk partials.
struct AttnArgs {
  const float* q;          // raw or prepared queries [qh*hd]
  const float* k_new;      // [kvh*hd]
  const float* v_new;      // [kvh*hd]
  const void* k_cache;     // [kvh][cap][hd]
  const void* v_cache;
  uint16_t* k_cache_w;     // if non-null: append new K/V (bf16) at position n
  uint16_t* v_cache_w;
  const float* q_norm;     // if non-null: apply (1+w) head RMSNorm to q and k
  const float* k_norm;
  const float* rope_freq;  // if non-null: [rotary/2] inverse frequencies
  const uint32_t* dev_pos; // position / cached count read on the device (graphs)
  uint32_t position;       // used when dev_pos is null
  uint32_t cached;         // used when dev_pos is null
  uint32_t qh, kvh, hd, cap, rotary;
  float eps;
  int cache_bf16;
  float* part;             // scratch: chunks * qh * (hd + 2) floats
  float* out;              // [qh*hd]
  uint32_t chunk;          // tokens per split (generic kernel)
  int* err;                // device error word for timed-out waits (may be null)
  // row-sharded model (xatt.n > 0): the merge stores this rank's output rows
  // and its gate rows (gate_in, [qh*hd]) as exchange words and gathers every
  // rank's into xatt.y / xgate.y (peer_exchange.cuh), instead of writing out
  PeerOut xatt, xgate;
  const float* gate_in;
};
// Longest cache (cached tokens + 1) the attention entry points accept: the
// generic kernel's 256-token chunks times the merge kernel's split limit.
constexpr uint64_t kAttnMaxTokens = uint64_t(4096) * 256;
// Scratch floats the split-K attention needs for a given cache size (an upper
// bound over both kernels launch_attention may pick).
uint64_t attn_scratch_floats(uint32_t qh, uint32_t kvh, uint32_t hd, uint32_t total_tokens,
                             uint32_t chunk);
void launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl);
void launch_rope(const float* x, const float* freq, uint32_t heads, uint32_t hd, uint32_t pos,
                 float* out, cudaStream_t s);

// All-gather over NVLink peer memory between the ranks' scratch blocks (mapped
// with CUDA IPC): every rank stores its slice of one or two vectors straight
// into every rank's receive buffers (same offsets in every block), then
// raises its flag in each block with a system-scope release; the kernel ends
// once this rank has seen every peer's flag reach `epoch` (bounded wait; a
// timeout sets KERR_TIMEOUT_FULL).
constexpr int kP2PMaxRanks = 8;
struct P2PGather {
  uint8_t* block[kP2PMaxRanks];  // every rank's scratch block, mapped here
  const float* send[2];
  uint64_t recv_off[2];          // byte offsets of the receive vectors in a block
  uint32_t count[2];             // floats per rank (count[1] = 0: one vector)
  uint32_t n, rank, epoch;
  uint64_t flag_off;             // byte offset of the flag words (64 B per rank)
  int* err;
  long long wait_cycles;         // bound of the wait for the other ranks (0: kWaitCycles)
};
void launch_p2p_allgather(const P2PGather& g, cudaStream_t s);

// Greedy argmax (runtime.rs:4301-4309). `key` is one device u64 scratch word;
// *index receives the index (0xFFFFFFFF when no finite value exists).
void launch_argmax(const float* v, uint64_t n, unsigned long long* key, uint32_t* index,
                   cudaStream_t s);

// Per-rank argmax key (global index = base + i) and the max over gathered keys.
void launch_argmax_key(const float* v, uint64_t n, uint32_t base, unsigned long long* key,
                       cudaStream_t s);
void launch_argmax_finish(unsigned long long* keys, uint32_t count, uint32_t* index,
                          cudaStream_t s);
// F32 matvecs whose input is the (1+w) RMSNorm of x, for one or two weight
// matrices of `rows` rows sharing x (the alpha and beta projections).
void launch_f32_matvec_norm2(const float* w0, float* y0, const float* w1, float* y1, uint32_t rows, uint32_t cols,
                             const float* x, const float* norm_w, float eps, cudaStream_t s);
// Dequantize Q4_K embedding row `*d_token` if it lies in [row_lo, row_hi), else zeros.
void launch_embed(const uint8_t* table, uint32_t cols, const uint32_t* d_token, uint32_t row_lo,
                  uint32_t row_hi, float* out, cudaStream_t s);
// Inverse RoPE frequencies computed on the host.
}  // namespace si
#include <vector>
namespace si {
void rope_freqs(float theta, uint32_t dims, std::vector<float>* out);

// Residual add y = a + b (length n).
void launch_add(const float* a, const float* b, float* y, uint64_t n, cudaStream_t s);
// y = silu(g) * u (length n): the MLP when gate and up differ in type.
void launch_swiglu(const float* g, const float* u, float* y, uint64_t n, cudaStream_t s);
// out[k][i] = a[k][i] / (1 + exp(-gate[k][i])) for k < batch, i < n.
void launch_siggate_many(const float* a, uint64_t lda, const float* gate, uint64_t ldg, float* out, uint64_t ldo,
                         uint32_t n, uint32_t batch, cudaStream_t s);

}  // namespace si
