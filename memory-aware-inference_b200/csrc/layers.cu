// Whole token mixers of one decoder layer on device buffers: the Gated
// DeltaNet mixer (gdn_token_mixer, src/qwen35_runtime.rs:409-624) and the
// full-attention mixer (attention_token_mixer, src/qwen35_runtime.rs:628-867).
//
// Both take the mixer input (the attn_norm output of the decoder block) and
// write the mixer output; the residual add stays with the caller, as in the
// reference's decoder block (qwen35_runtime.rs:1329-1387). They run the same
// kernels as the model's layer bodies:
//  * GDN: one grouped matvec for qkv and z, the alpha/beta F32 projections
//    (unless the gates are supplied), gdn_layer_kernel (conv + L2 norms +
//    head repeat + gates + recurrence), and ssm_out with the gated RMSNorm
//    as its x prologue.
//  * Attention: one grouped matvec for q (queries and output gate), k and v;
//    the split-K attention kernel with the q/k (1+w) head norm, partial RoPE
//    and the append of the new key/value to the bf16 cache fused in; o-proj
//    with the sigmoid output gate as its x prologue.
// Every buffer, the caller's workspace included, is device memory; the work
// is enqueued on the given stream and nothing is allocated or synchronised.
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "common.cuh"
#include "ctx.h"
#include "kernels.cuh"
#include "qmatvec.cuh"

using namespace si;

namespace {

bool is_kquant(uint32_t t) { return block_bytes_of(t) != 0; }

// A grouped matvec over segments sharing x: one launch when all types agree,
// else one launch per segment.
int group_matvec(si_ctx* ctx, QmvParams p, const uint32_t* types, cudaStream_t s) {
  bool same = true;
  for (uint32_t i = 1; i < p.nseg; ++i) same = same && types[i] == types[0];
  std::string msg;
  if (same) {
    p.type = types[0];
    const int rc = launch_qmv(p, s, ctx->sm_count, true, &msg);
    return rc ? fail(ctx, rc, msg) : SI_OK;
  }
  for (uint32_t i = 0; i < p.nseg; ++i) {
    QmvParams q = p;
    q.nseg = 1;
    q.seg[0] = p.seg[i];
    q.items = p.seg[i].rows;
    q.type = types[i];
    if (int rc = launch_qmv(q, s, ctx->sm_count, true, &msg)) return fail(ctx, rc, msg);
  }
  return SI_OK;
}

int check_gdn(si_ctx* ctx, const si_gdn_layer_desc* d) {
  if (!d) return fail(ctx, SI_E_INVALID, "null GDN layer description");
  if (d->hidden == 0 || d->hidden % 256 || d->hidden > kQmvMaxCols)
    return fail(ctx, SI_E_INVALID, "GDN layer hidden width must be a positive multiple of 256");
  if (d->head_dim != 128)
    return fail(ctx, SI_E_UNSUPPORTED, "GDN layer head_dim must be 128");
  if (d->key_heads == 0 || d->value_heads == 0 || d->value_heads % d->key_heads ||
      (uint64_t(d->value_heads) * 128) % 256 || d->value_heads > 4096)
    return fail(ctx, SI_E_INVALID, "GDN layer head counts are invalid");
  if (d->conv_kernel < 2 || d->conv_kernel > 8)
    return fail(ctx, SI_E_UNSUPPORTED, "GDN layer conv kernel must be 2..8");
  if (!is_kquant(d->qkv_type) || !is_kquant(d->z_type) || !is_kquant(d->out_type))
    return fail(ctx, SI_E_UNSUPPORTED, "GDN layer projections must be Q4_K, Q5_K or Q6_K");
  if (!d->qkv || !d->z || !d->out || !d->conv || !d->norm)
    return fail(ctx, SI_E_INVALID, "GDN layer weights are null");
  return SI_OK;
}

int check_attn(si_ctx* ctx, const si_attention_layer_desc* d) {
  if (!d) return fail(ctx, SI_E_INVALID, "null attention layer description");
  if (d->hidden == 0 || d->hidden % 256 || d->hidden > kQmvMaxCols)
    return fail(ctx, SI_E_INVALID, "attention layer hidden width must be a positive multiple of 256");
  if (d->query_heads == 0 || d->kv_heads == 0 || d->query_heads % d->kv_heads || d->head_dim == 0 ||
      d->head_dim % 32)
    return fail(ctx, SI_E_INVALID, "attention layer head dimensions are invalid");
  if (d->head_dim > 256 || d->query_heads / d->kv_heads > 8)
    return fail(ctx, SI_E_UNSUPPORTED, "attention head_dim > 256 or GQA group > 8 is not supported");
  if ((uint64_t(d->query_heads) * d->head_dim) % 256 || (uint64_t(d->kv_heads) * d->head_dim) % 16)
    return fail(ctx, SI_E_UNSUPPORTED, "attention layer widths must allow K-quant rows");
  if (d->rotary_dim % 2 || d->rotary_dim > d->head_dim)
    return fail(ctx, SI_E_INVALID, "attention rotary width is invalid");
  if (!is_kquant(d->q_type) || !is_kquant(d->k_type) || !is_kquant(d->v_type) || !is_kquant(d->o_type))
    return fail(ctx, SI_E_UNSUPPORTED, "attention layer projections must be Q4_K, Q5_K or Q6_K");
  if (!d->q || !d->k || !d->v || !d->o || !d->q_norm || !d->k_norm)
    return fail(ctx, SI_E_INVALID, "attention layer weights are null");
  return SI_OK;
}

uint64_t gdn_work(const si_gdn_layer_desc* d) {
  const uint64_t vw = uint64_t(d->value_heads) * 128, proj = 2ull * d->key_heads * 128 + vw;
  return proj + 2 * vw + 2ull * d->value_heads;
}

// qg [2 qw] | k [kvw] | v [kvw] | att [qw] | rope [rotary/2, padded to 4] | split-K partials
uint64_t attn_work(const si_attention_layer_desc* d, uint64_t cached) {
  const uint64_t qw = uint64_t(d->query_heads) * d->head_dim, kvw = uint64_t(d->kv_heads) * d->head_dim;
  return 3 * qw + 2 * kvw + ((d->rotary_dim / 2 + 3) & ~3ull) +
         attn_scratch_floats(d->query_heads, d->kv_heads, d->head_dim, uint32_t(cached + 1), 256);
}

}  // namespace

extern "C" {

uint64_t si_gdn_layer_workspace_floats(const si_gdn_layer_desc* d) { return d ? gdn_work(d) : 0; }

uint64_t si_attention_layer_workspace_floats(const si_attention_layer_desc* d, uint64_t cached_tokens) {
  if (!d || cached_tokens + 1 > kAttnMaxTokens || d->kv_heads == 0) return 0;
  return attn_work(d, cached_tokens);
}

int si_gdn_layer_dev(si_ctx* ctx, const si_gdn_layer_desc* d, const float* x, const float* conv_state_in,
                     float* conv_state_out, float* state, const float* gates, float* out, float* work,
                     void* stream) {
  if (!ctx) return SI_E_INVALID;
  if (int rc = check_gdn(ctx, d)) return rc;
  if (!x || !conv_state_in || !conv_state_out || !state || !out || !work)
    return fail(ctx, SI_E_INVALID, "GDN layer buffers are null");
  if (conv_state_in == conv_state_out)
    return fail(ctx, SI_E_INVALID, "GDN layer conv state must be read and written through different buffers");
  if (!gates && (!d->alpha || !d->beta || !d->a_log || !d->dt_bias))
    return fail(ctx, SI_E_INVALID, "GDN layer needs the alpha/beta projections or supplied gates");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(work)) & 15)
    return fail(ctx, SI_E_INVALID, "GDN layer input and workspace must be 16-byte aligned");
  const cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const uint32_t kh = d->key_heads, vh = d->value_heads, H = uint32_t(d->hidden);
  const uint32_t vw = vh * 128, proj = 2 * kh * 128 + vw;
  float* qkv = work;
  float* z = qkv + proj;
  float* core = z + vw;
  float* ab = core + vw;
  QmvParams p = {};
  p.cols = H;
  p.nseg = 2;
  p.seg[0] = {static_cast<const uint8_t*>(d->qkv), qkv, nullptr, proj, 0};
  p.seg[1] = {static_cast<const uint8_t*>(d->z), z, nullptr, vw, 0};
  p.items = proj + vw;
  p.xmode = XM_RAW;
  p.x = x;
  p.eps = d->epsilon;
  p.err = ctx->d_err;
  si::qscratch_for(ctx, s, &p.scratch, &p.scratch_bytes);
  const uint32_t types[2] = {d->qkv_type, d->z_type};
  if (int rc = group_matvec(ctx, p, types, s)) return rc;
  if (!gates) {
    launch_f32_matvec(d->alpha, vh, H, x, ab, s);
    launch_f32_matvec(d->beta, vh, H, x, ab + vh, s);
  }
  GdnLayerArgs g = {};
  g.qkv = qkv;
  g.conv_w = d->conv;
  g.conv_in = conv_state_in;
  g.conv_out = conv_state_out;
  g.state = state;
  g.gates = gates;
  g.alpha = ab;
  g.beta_logit = ab + vh;
  g.a_log = d->a_log;
  g.dt_bias = d->dt_bias;
  g.core = core;
  g.key_heads = kh;
  g.value_heads = vh;
  g.kernel = d->conv_kernel;
  launch_gdn_layer(g, s, false);
  QmvParams o = {};
  o.type = d->out_type;
  o.cols = vw;
  o.nseg = 1;
  o.seg[0] = {static_cast<const uint8_t*>(d->out), out, nullptr, H, 0};
  o.items = H;
  o.xmode = XM_GATED;
  o.x = core;
  o.xaux = z;
  o.xw = d->norm;
  o.head_dim = 128;
  o.eps = d->epsilon;
  o.err = ctx->d_err;
  si::qscratch_for(ctx, s, &o.scratch, &o.scratch_bytes);
  std::string msg;
  if (int rc = launch_qmv(o, s, ctx->sm_count, true, &msg)) return fail(ctx, rc, msg);
  if (cudaError_t e = cudaGetLastError()) return cuda_fail(ctx, e, "GDN layer launch");
  note_async_submission(ctx);
  return SI_OK;
}

int si_attention_layer_dev(si_ctx* ctx, const si_attention_layer_desc* d, const float* x, uint64_t position,
                           uint16_t* key_cache, uint16_t* value_cache, uint64_t cached_tokens,
                           uint64_t capacity_tokens, float* out, float* work, void* stream) {
  if (!ctx) return SI_E_INVALID;
  if (int rc = check_attn(ctx, d)) return rc;
  if (!x || !key_cache || !value_cache || !out || !work)
    return fail(ctx, SI_E_INVALID, "attention layer buffers are null");
  if (capacity_tokens > 0xffffffffull || cached_tokens >= capacity_tokens)
    return fail(ctx, SI_E_STATE, "full-attention KV cache capacity exhausted");
  if (cached_tokens + 1 > kAttnMaxTokens || position > 0xffffffffull)
    return fail(ctx, SI_E_UNSUPPORTED, "attention over more than 1048576 tokens is not supported");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(work)) & 15)
    return fail(ctx, SI_E_INVALID, "attention layer input and workspace must be 16-byte aligned");
  const cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const uint32_t qh = d->query_heads, kvh = d->kv_heads, hd = d->head_dim, H = uint32_t(d->hidden);
  const uint32_t qw = qh * hd, kvw = kvh * hd;
  float* qg = work;
  float* kk = qg + 2 * qw;
  float* vv = kk + kvw;
  float* att = vv + kvw;
  float* rope = att + qw;
  float* part = rope + ((d->rotary_dim / 2 + 3) & ~3u);
  if (d->rotary_dim) {
    std::vector<float> f;
    rope_freqs(d->rope_theta, d->rotary_dim, &f);
    if (cudaError_t e = cudaMemcpyAsync(rope, f.data(), f.size() * 4, cudaMemcpyHostToDevice, s))
      return cuda_fail(ctx, e, "attention layer rope table");
  }
  QmvParams p = {};
  p.cols = H;
  p.nseg = 3;
  p.seg[0] = {static_cast<const uint8_t*>(d->q), qg, nullptr, 2 * qw, 0};
  p.seg[1] = {static_cast<const uint8_t*>(d->k), kk, nullptr, kvw, 0};
  p.seg[2] = {static_cast<const uint8_t*>(d->v), vv, nullptr, kvw, 0};
  p.items = 2 * qw + 2 * kvw;
  p.xmode = XM_RAW;
  p.x = x;
  p.eps = d->epsilon;
  p.err = ctx->d_err;
  si::qscratch_for(ctx, s, &p.scratch, &p.scratch_bytes);
  const uint32_t types[3] = {d->q_type, d->k_type, d->v_type};
  if (int rc = group_matvec(ctx, p, types, s)) return rc;
  AttnArgs a = {};
  a.q = qg;
  a.k_new = kk;
  a.v_new = vv;
  a.k_cache = key_cache;
  a.v_cache = value_cache;
  a.k_cache_w = key_cache;
  a.v_cache_w = value_cache;
  a.q_norm = d->q_norm;
  a.k_norm = d->k_norm;
  a.rope_freq = d->rotary_dim ? rope : nullptr;
  a.position = uint32_t(position);
  a.cached = uint32_t(cached_tokens);
  a.qh = qh;
  a.kvh = kvh;
  a.hd = hd;
  a.cap = uint32_t(capacity_tokens);
  a.rotary = d->rotary_dim;
  a.eps = d->epsilon;
  a.cache_bf16 = 1;
  a.part = part;
  a.out = att;
  a.chunk = 256;
  a.err = ctx->d_err;
  launch_attention(a, s, true);
  QmvParams o = {};
  o.type = d->o_type;
  o.cols = qw;
  o.nseg = 1;
  o.seg[0] = {static_cast<const uint8_t*>(d->o), out, nullptr, H, 0};
  o.items = H;
  o.xmode = XM_SIGGATE;
  o.x = att;
  o.xaux = qg + qw;
  o.eps = d->epsilon;
  o.err = ctx->d_err;
  si::qscratch_for(ctx, s, &o.scratch, &o.scratch_bytes);
  std::string msg;
  if (int rc = launch_qmv(o, s, ctx->sm_count, true, &msg)) return fail(ctx, rc, msg);
  if (cudaError_t e = cudaGetLastError()) return cuda_fail(ctx, e, "attention layer launch");
  note_async_submission(ctx);
  return SI_OK;
}

}  // extern "C"
