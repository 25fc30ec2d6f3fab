/* si_cuda.h — C ABI of the B200 (sm_100a) batch-1 K-quant decode backend.
 *
 * This is the drop-in boundary that replaces the Metal backend
 * (`MetalContext`, src/metal.rs) of vrlda/memory-aware-inference on the
 * batch-1 decode hot path. Every entry point names the reference method it
 * replaces (file:line inside the reference project). A Rust FFI crate binds
 * these symbols one-to-one and keeps the reference's
 * `Result<Vec<f32>, String>` surface: a non-zero status maps to `Err` with the
 * text of si_last_error().
 *
 * Conventions
 *  - Every function returns an int status: SI_OK (0) or a negative SI_E_*.
 *  - Plain pointers are HOST memory unless the function name ends in `_dev`;
 *    `_dev` functions take device pointers and a cudaStream_t (passed as
 *    void*), enqueue work and return without synchronising.
 *  - Host-memory entry points are synchronous, like the reference's
 *    commit-and-wait calls (metal.rs:2320-2337): inputs are copied in, the
 *    kernel runs, outputs are copied back before the call returns.
 *  - One context serves one compute thread plus any number of threads that
 *    upload weights (metal.rs:2585-2640 are called from staging workers);
 *    uploads are internally serialised.
 */
#ifndef SI_CUDA_H
#define SI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define SI_OK 0
#define SI_E_INVALID (-1)  /* shape / length / argument validation failed */
#define SI_E_CUDA (-2)     /* a CUDA runtime call failed */
#define SI_E_NOMEM (-3)    /* device or pinned allocation failed */
#define SI_E_BUDGET (-4)   /* plan does not fit the HBM budget */
#define SI_E_TIMEOUT (-5)  /* a bounded device or host wait gave up */
#define SI_E_COMM (-6)     /* NCCL failure */
#define SI_E_STATE (-7)    /* object used in the wrong state (e.g. KV full) */
#define SI_E_UNSUPPORTED (-8)

/* ---- GGML tensor types (quant.rs:8-16) ---------------------------------- */
#define SI_GGML_TYPE_F32 0u
#define SI_GGML_TYPE_Q4_K 12u
#define SI_GGML_TYPE_Q5_K 13u
#define SI_GGML_TYPE_Q6_K 14u

typedef struct si_ctx si_ctx;
typedef struct si_weight si_weight;
typedef struct si_model si_model;

/* Context configuration: one explicit struct instead of the reference's
 * SI_* environment variables (qwen35_runtime.rs:1788-1793, 2288-2293). */
typedef struct si_ctx_config {
  uint64_t hbm_budget_bytes; /* bound for model weights+ring+state; 0 = no bound */
  uint32_t stage_depth;      /* staging-ring depth: default 3, clamped to 1..4 */
  uint32_t flags;            /* SI_CTX_FLAG_* bits, 0 = defaults */
} si_ctx_config;
/* Row-sharded models exchange their sharded vectors over NVLink peer memory
 * (CUDA IPC mappings of the ranks' scratch) by default; this flag keeps every
 * exchange on NCCL collectives instead. */
#define SI_CTX_FLAG_NCCL_COLLECTIVES 1u

/* ---- context (MetalContext::new, metal.rs:2170) ------------------------- */
int si_ctx_create(int device, const si_ctx_config* cfg, si_ctx** out);
void si_ctx_destroy(si_ctx* ctx);
/* Text of the last error on this context (the reference's Err(String)). */
const char* si_last_error(const si_ctx* ctx);
/* Text of the last error of a call that had no context (si_ctx_create). */
const char* si_global_last_error(void);
/* metal::probe (metal.rs:18-24, 1770-1779): the device's name, its memory
 * (the working-set bound: total HBM bytes), the SM count, the compute
 * capability and the number of visible devices. No context needed. */
typedef struct si_device_info {
  char name[256];
  uint64_t total_bytes;
  uint32_t sm_count, cc_major, cc_minor, device_count;
} si_device_info;
int si_device_probe(int device, si_device_info* out);
/* Number of SMs and the device ordinal the context runs on. */
int si_ctx_info(const si_ctx* ctx, int* device, int* sm_count);
/* The context's compute stream (cudaStream_t as void*). */
void* si_ctx_stream(si_ctx* ctx);

/* ---- telemetry (metal.rs:2312-2445) ------------------------------------- */
typedef struct si_stats {
  uint64_t current_allocated_bytes;
  uint64_t peak_allocated_bytes;     /* peak_allocated_bytes, metal.rs:2339 */
  uint64_t peak_active_weight_bytes; /* metal.rs:2343 */
  uint64_t peak_kv_bytes;            /* metal.rs:2347 */
  uint64_t peak_scratch_bytes;       /* metal.rs:2351 */
  uint64_t submitted;                /* command_stats, metal.rs:2316 */
  uint64_t waited;
  uint64_t wait_nanos;
  uint64_t async_submitted;          /* `_dev` enqueues (also counted in submitted) */
} si_stats;
int si_get_stats(const si_ctx* ctx, si_stats* out);
/* CommandStatsSnapshot::delta_since (metal.rs:1891-1947): the command
 * counters (submitted, async_submitted, waited, wait_nanos) of `after` minus
 * those of `before`, saturating at 0; the byte fields are `after`'s. */
int si_stats_delta(const si_stats* after, const si_stats* before, si_stats* out);
int si_reset_peaks(si_ctx* ctx);
/* Host-side fault injection for tests of the failure paths (the reference
 * turns every such failure into Err(String); no GPU fault is involved). The
 * call at `site` that follows `skip` further calls there fails once, as the
 * real call fails: an allocation with SI_E_NOMEM, a file read as a short
 * read. Process-wide; site 0 disarms every site. */
#define SI_FAULT_PINNED_ALLOC 1u /* pinned host memory of a model's weights */
#define SI_FAULT_DEVICE_ALLOC 2u /* device memory: weights, staged layers, models, snapshots */
#define SI_FAULT_FILE_READ 3u    /* GGUF header reads and payload preads */
int si_fault_inject(uint32_t site, uint32_t skip);
/* sample_allocated (metal.rs:2374-2378): fold the current allocation into the peak. */
int si_sample_allocated(si_ctx* ctx); /* reset_peaks, metal.rs:2358 */

/* ---- weights (QuantWeight, metal.rs:1840-1846) -------------------------- */
/* upload_quant_weight_private (metal.rs:2502): copy bytes into device memory. */
int si_weight_upload(si_ctx* ctx, const void* host, uint64_t bytes, uint32_t ggml_type,
                     si_weight** out);
/* bind_quant_weight_mapped (metal.rs:2549): keep the bytes in (registered,
 * pinned) host memory; each use streams them to the device first. The host
 * bytes must outlive the handle (metal.rs:2614-2617). */
int si_weight_bind_host(si_ctx* ctx, const void* host, uint64_t bytes, uint32_t ggml_type,
                        si_weight** out);
void si_weight_free(si_weight* w);
uint64_t si_weight_bytes(const si_weight* w);   /* QuantWeight::byte_len */
uint32_t si_weight_type(const si_weight* w);    /* QuantWeight::ggml_type */
const void* si_weight_device_ptr(const si_weight* w); /* NULL for host-bound */

/* ---- lossless dequant (quant.rs:18-174), parity use --------------------- */
int si_dequantize(si_ctx* ctx, uint32_t ggml_type, const void* bytes, uint64_t nbytes,
                  uint64_t elements, float* out);
int si_dequantize_dev(si_ctx* ctx, uint32_t ggml_type, const void* bytes_dev,
                      uint64_t elements, float* out_dev, void* stream);
/* q4_k_embedding_row (metal.rs:3734): dequantize one Q4_K row. */
int si_q4_k_embedding_row(si_ctx* ctx, const void* row_bytes, uint64_t nbytes,
                          uint64_t columns, float* out);

/* ---- K-quant matvec: y = W x, W row-major GGUF super-blocks -------------- */
/* gguf_quant_matvec_bytes (metal.rs:4000); q4_k_matvec / q5_k_matvec /
 * q6_k_matvec (metal.rs:3357, 4307, 4325) are this call with a fixed type. */
int si_gguf_quant_matvec_bytes(si_ctx* ctx, uint32_t ggml_type, const void* w, uint64_t nbytes,
                               uint64_t rows, uint64_t cols, const float* x, float* y);
int si_q4_k_matvec(si_ctx* ctx, const void* w, uint64_t nbytes, uint64_t rows, uint64_t cols,
                   const float* x, float* y);
int si_q5_k_matvec(si_ctx* ctx, const void* w, uint64_t nbytes, uint64_t rows, uint64_t cols,
                   const float* x, float* y);
int si_q6_k_matvec(si_ctx* ctx, const void* w, uint64_t nbytes, uint64_t rows, uint64_t cols,
                   const float* x, float* y);
/* gguf_quant_matvec_weight (metal.rs:3923). */
int si_gguf_quant_matvec_weight(si_ctx* ctx, const si_weight* w, uint64_t rows, uint64_t cols,
                                const float* x, float* y);
/* gguf_quant_matvec_many_weights (metal.rs:4652): n <= 4 matrices, one x. */
int si_gguf_quant_matvec_many_weights(si_ctx* ctx, uint32_t n, const si_weight* const* w,
                                      const uint64_t* rows, const uint64_t* cols,
                                      const float* x, float* const* y);
/* Device form: `w_dev` holds rows*cols/256 blocks of `ggml_type`.
 * Calls of the device forms on one context may run on different streams at
 * once: a Q6_K matvec of 2,048+ rows (or 64+ blocks per row) finishes the row
 * groups it shares between CTAs in a scratch slot of the context that belongs
 * to the launching stream (8 slots; past the eighth stream a call runs
 * without one, slower). A CUDA graph that captured such a call keeps the
 * capture stream's slot: replay it on that stream, or not at the same time
 * as other calls on that stream. */
int si_qmatvec_dev(si_ctx* ctx, uint32_t ggml_type, const void* w_dev, uint64_t rows,
                   uint64_t cols, const float* x_dev, float* y_dev, void* stream);
/* Batched matvec for up to 8 inputs with one traversal of the weights
 * (gguf_quant_matmul_many_bytes / _weight, metal.rs:4067-4230; kernels
 * si_q{4,5,6}_k_matmul_many, metal.rs:1055-1267). inputs: batch x cols f32,
 * candidate-major; outputs: batch x rows f32, candidate-major. */
int si_gguf_quant_matmul_many_bytes(si_ctx* ctx, uint32_t ggml_type, const void* weights, uint64_t nbytes,
                                    uint64_t rows, uint64_t cols, uint64_t batch, const float* inputs,
                                    float* outputs);
int si_gguf_quant_matmul_many_weight(si_ctx* ctx, const si_weight* weight, uint64_t rows, uint64_t cols,
                                     uint64_t batch, const float* inputs, float* outputs);
/* Device-pointer form on `stream` (NULL: the context's stream). Its
 * tensor-core scratch (digits, scales, panel sums) is the context's: calls on
 * one context must not overlap on the GPU. */
int si_qmatmul_many_dev(si_ctx* ctx, uint32_t ggml_type, const void* weights_dev, uint64_t rows, uint64_t cols,
                        uint64_t batch, const float* x_dev, float* y_dev, void* stream);
/* f32_matvec (metal.rs:2983). */
int si_f32_matvec(si_ctx* ctx, const float* w, uint64_t rows, uint64_t cols, const float* x,
                  float* y);

/* ---- staged layers (metal.rs:1852-1869, 2585-2637) ------------------------ */
/* A packed decoder layer: upload_staged_qwen_layer_private copies it to device
 * memory once (each named range at its own 256-byte aligned offset, so every
 * view meets the kernels' alignment); bind_staged_qwen_layer_shared keeps it in
 * the caller's host memory (page-locked when possible; the bytes must outlive
 * the layer). Ranges: name -> [start, end) in the packed bytes. Views from
 * si_staged_layer_weight (PrivateStagedQwenLayer::quant_weight) are freed with
 * si_weight_free before the layer. */
typedef struct si_staged_layer si_staged_layer;
int si_staged_layer_upload(si_ctx* ctx, const void* packed, uint64_t bytes, uint32_t n_ranges,
                           const char* const* names, const uint64_t* starts, const uint64_t* ends,
                           si_staged_layer** out);
int si_staged_layer_bind_host(si_ctx* ctx, const void* packed, uint64_t bytes, uint32_t n_ranges,
                              const char* const* names, const uint64_t* starts, const uint64_t* ends,
                              si_staged_layer** out);
int si_staged_layer_weight(const si_staged_layer* layer, const char* name, uint32_t ggml_type, si_weight** out);
void si_staged_layer_free(si_staged_layer* layer);
/* gguf_quant_matvec_many_bytes (metal.rs:4878): n matrices of any K-quant type
 * sharing x (cols columns). */
int si_gguf_quant_matvec_many_bytes(si_ctx* ctx, uint32_t n, const uint32_t* ggml_types,
                                    const void* const* weights, const uint64_t* nbytes, const uint64_t* rows,
                                    uint64_t cols, const float* x, float* const* y);
/* f32_matvec_many_gguf_tensors (metal.rs:4780): n F32 matrices sharing x. */
int si_f32_matvec_many(si_ctx* ctx, uint32_t n, const float* const* weights, const uint64_t* rows, uint64_t cols,
                       const float* x, float* const* y);

/* ---- fused SwiGLU (metal.rs:3402-3732) ----------------------------------- */
/* q4_k_fused_gate_up (metal.rs:3402): out = SiLU(G x) * (U x). */
int si_q4_k_fused_gate_up(si_ctx* ctx, const void* gate, const void* up, uint64_t nbytes,
                          uint64_t rows, uint64_t cols, const float* x, float* out);
/* q4_k_fused_gate_up_weights (metal.rs:3489). */
int si_q4_k_fused_gate_up_weights(si_ctx* ctx, const si_weight* gate, const si_weight* up,
                                  uint64_t rows, uint64_t cols, const float* x, float* out);
/* gguf_quant_fused_mlp_weights (metal.rs:3569): y = D (SiLU(G x) * (U x)). */
int si_gguf_quant_fused_mlp_weights(si_ctx* ctx, const si_weight* gate, const si_weight* up,
                                    const si_weight* down, uint64_t gate_rows, uint64_t cols,
                                    uint64_t down_rows, const float* x, float* y);
int si_fused_gate_up_dev(si_ctx* ctx, uint32_t ggml_type, const void* gate_dev,
                         const void* up_dev, uint64_t rows, uint64_t cols, const float* x_dev,
                         float* out_dev, void* stream);
int si_fused_mlp_dev(si_ctx* ctx, uint32_t gate_type, const void* gate_dev, const void* up_dev,
                     uint32_t down_type, const void* down_dev, uint64_t inter, uint64_t hidden,
                     const float* x_dev, float* act_dev, float* y_dev, void* stream);

/* ---- Gated DeltaNet primitives (qwen35.rs, metal.rs:3122-3352) ----------- */
/* gated_delta_step (metal.rs:3122): state [heads][key_dim][value_dim]. */
int si_gated_delta_step(si_ctx* ctx, const float* q, const float* k, const float* v,
                        const float* gate, const float* beta, const float* state_in,
                        uint64_t heads, uint64_t key_dim, uint64_t value_dim, float* out,
                        float* state_out);
/* causal_conv1d_step (metal.rs:3263): state [channels][kernel-1], chronological. */
int si_causal_conv1d_step(si_ctx* ctx, const float* x, const float* state_in, const float* w,
                          uint64_t channels, uint64_t kernel, float* out, float* state_out);
/* rms_norm_gated (metal.rs:2773) and rms_norm_heads (metal.rs:2856). */
int si_rms_norm_gated(si_ctx* ctx, const float* x, const float* gate, const float* w,
                      uint64_t heads, uint64_t head_dim, float eps, float* out);
int si_rms_norm_heads(si_ctx* ctx, const float* x, const float* w, uint64_t heads,
                      uint64_t head_dim, float eps, float* out);

/* ---- attention (metal.rs:6860-7083) -------------------------------------- */
/* rope (metal.rs:6860): adjacent-pair rotation over the whole head_dim. */
int si_rope(si_ctx* ctx, const float* x, uint64_t heads, uint64_t head_dim, uint64_t position,
            float theta, float* out);
#define SI_CACHE_F32 0
#define SI_CACHE_BF16 1
/* AttentionDecodeInput (metal.rs:27-38) plus the cache element type. */
typedef struct si_attention_decode_input {
  const float* query;      /* [query_heads * head_dim] */
  const void* key_cache;   /* [kv_heads][capacity][head_dim], f32 or bf16 bits */
  const void* value_cache;
  const float* new_keys;   /* [kv_heads * head_dim] current token, f32 */
  const float* new_values;
  uint64_t query_heads, key_value_heads, head_dim, cached_tokens, cache_capacity_tokens;
  int cache_type;          /* SI_CACHE_F32 or SI_CACHE_BF16 */
} si_attention_decode_input;
/* attention_decode (metal.rs:6915). */
int si_attention_decode(si_ctx* ctx, const si_attention_decode_input* in, float* out);

/* Allocation-free form of si_attention_decode for callers that cannot
 * allocate device memory at call time (for example while a stream is being
 * captured, or under a runtime that forbids cudaMalloc after start-up). No
 * counterpart in the reference. All pointers inside `in` and `out` are
 * DEVICE pointers; the work is enqueued on `stream` (cudaStream_t as void*,
 * NULL = legacy default stream) and the call returns without synchronising.
 * The split-K partials use a fixed 4 MiB array built into the library on every
 * GPU that loads it: calls needing more (qh * (hd + 2) floats per split; at
 * most max(ceil((n+1)/256), min(ceil(n/64), 148/kvh)) splits for n cached
 * tokens) fail with SI_E_UNSUPPORTED. Calls share that array, so calls
 * that overlap on the GPU race. The first call on a device looks up the
 * array's address; make it before any stream capture (a first call during a
 * capture fails with SI_E_UNSUPPORTED). A split whose bounded wait for K/V
 * tiles runs out (about 2 s) contributes nothing and sets a device error
 * word; a later call made outside a capture, on a stream that has drained,
 * returns SI_E_TIMEOUT for it and clears the word. Errors are reported
 * through si_global_last_error(). */
int si_attention_decode_noalloc_dev(const si_attention_decode_input* in, float* out, void* stream);

/* ---- whole token mixers of one decoder layer (device buffers) ----------- */
/* The Gated DeltaNet token mixer of one layer (gdn_token_mixer,
 * qwen35_runtime.rs:409-624): qkv and z projections of x, causal conv + SiLU,
 * q/k L2 norms, key-head repeat, the gates, the recurrent update, the gated
 * RMSNorm (w, not 1+w) and ssm_out. x is the mixer input (the block's
 * attn_norm output); `out` receives the mixer output without the residual.
 * Matrices are [rows][cols] GGUF K-quant rows; F32 tensors row-major. */
typedef struct si_gdn_layer_desc {
  uint64_t hidden;                 /* x / out width, a multiple of 256 */
  uint32_t key_heads, value_heads; /* value head h uses key head h / (value_heads / key_heads) */
  uint32_t head_dim;               /* 128 */
  uint32_t conv_kernel;            /* 2..8 */
  float epsilon;                   /* gated RMSNorm epsilon */
  const void* qkv; uint32_t qkv_type; /* [(2 kh + vh) * 128][hidden]: q | k | v channels */
  const void* z; uint32_t z_type;     /* [vh * 128][hidden] */
  const void* out; uint32_t out_type; /* [hidden][vh * 128] */
  const float* conv;               /* [(2 kh + vh) * 128][conv_kernel] */
  const float* norm;               /* [128] gated-norm weight */
  const float* alpha;              /* [vh][hidden]; these four are read only when gates == NULL */
  const float* beta;               /* [vh][hidden] */
  const float* a_log;              /* [vh] */
  const float* dt_bias;            /* [vh] */
} si_gdn_layer_desc;
/* Floats of device workspace si_gdn_layer_dev needs: (2 kh + vh) * 128 + 2 vh * 128 + 2 vh. */
uint64_t si_gdn_layer_workspace_floats(const si_gdn_layer_desc* desc);
/* Device pointers throughout; enqueued on `stream` (NULL = the context's
 * stream), nothing allocated or synchronised. conv_state_in/out are
 * [(2 kh + vh) * 128][conv_kernel - 1] (chronological) and must differ;
 * state is the f32 recurrent state [vh][128][128], updated in place. gates,
 * if not NULL, is [g[vh], beta[vh]] used as is (g = -softplus(...) already,
 * beta = sigmoid(...) already); else g and beta come from the alpha/beta
 * projections, a_log and dt_bias (qwen35_runtime.rs:577-601). x and work are
 * 16-byte aligned; work holds si_gdn_layer_workspace_floats(desc) floats. */
int si_gdn_layer_dev(si_ctx* ctx, const si_gdn_layer_desc* desc, const float* x, const float* conv_state_in,
                     float* conv_state_out, float* state, const float* gates, float* out, float* work,
                     void* stream);

/* The full-attention token mixer of one layer (attention_token_mixer,
 * qwen35_runtime.rs:628-867) over a bf16 head-major KV cache
 * [kv_heads][capacity][head_dim] (cache.rs:1-4): q (the first half of the q
 * projection; the second half is the output gate), k and v projections; (1+w)
 * head RMSNorm of q and k; partial RoPE on dims [0, rotary_dim) at `position`
 * (metal.rs:1655-1679); attention over the cached tokens plus the new one
 * (scores scaled by 1/sqrt(head_dim)); the new key and value appended at slot
 * cached_tokens; out = o-proj of (attention * sigmoid(gate)), no residual. */
typedef struct si_attention_layer_desc {
  uint64_t hidden;                 /* x / out width, a multiple of 256 */
  uint32_t query_heads, kv_heads, head_dim, rotary_dim;
  float rope_theta, epsilon;
  const void* q; uint32_t q_type;  /* [2 * qh * hd][hidden]: queries, then the gate */
  const void* k; uint32_t k_type;  /* [kvh * hd][hidden] */
  const void* v; uint32_t v_type;  /* [kvh * hd][hidden] */
  const void* o; uint32_t o_type;  /* [hidden][qh * hd] */
  const float* q_norm;             /* [hd] (1+w) */
  const float* k_norm;             /* [hd] (1+w) */
} si_attention_layer_desc;
/* Floats of device workspace si_attention_layer_dev needs with
 * `cached_tokens` tokens in the cache (0 when the arguments are invalid). */
uint64_t si_attention_layer_workspace_floats(const si_attention_layer_desc* desc, uint64_t cached_tokens);
/* Device pointers throughout; enqueued on `stream` (NULL = the context's
 * stream), nothing allocated or synchronised. cached_tokens < capacity_tokens
 * (SI_E_STATE otherwise). x and work are 16-byte aligned. */
int si_attention_layer_dev(si_ctx* ctx, const si_attention_layer_desc* desc, const float* x, uint64_t position,
                           uint16_t* key_cache, uint16_t* value_cache, uint64_t cached_tokens,
                           uint64_t capacity_tokens, float* out, float* work, void* stream);

/* ---- row-sharded matvec with the all-gather inside the kernel ----------- */
/* Row sharding of the matvec over the GPUs of one box is the BASELINE's
 * multi-GPU partitioning of gguf_quant_matvec_weight (metal.rs:3923); the
 * reference is single-GPU, so these have no reference counterpart.
 * A peer buffer: `bytes` of device memory on every rank of the context's
 * communicator (one rank without one), each rank's copy mapped into every
 * other rank (CUDA IPC over NVLink). Collective: every rank calls it with the
 * same size. Each rank's allocation also holds the in-kernel exchange's
 * words (two 8-byte words per float of the data) and its counters: about
 * five times `bytes` in all. */
typedef struct si_peer_buffer si_peer_buffer;
int si_peer_buffer_create(si_ctx* ctx, uint64_t bytes, si_peer_buffer** out);
/* A group of `nranks` buffers all on this context's GPU standing in for the
 * ranks, this process acting as rank `rank`: for testing the exchange on one
 * GPU. The other ranks never run, so a sharded matvec's wait for them runs out
 * after about wait_us microseconds (0 = the default of about 2 s) and the next
 * si_ctx_synchronize reports SI_E_TIMEOUT. */
int si_peer_buffer_create_local(si_ctx* ctx, uint64_t bytes, uint32_t nranks, uint32_t rank, uint64_t wait_us,
                                si_peer_buffer** out);
void si_peer_buffer_destroy(si_peer_buffer* buf);
/* This rank's copy (device pointer). */
void* si_peer_buffer_local(const si_peer_buffer* buf);
/* y = W x with W row-sharded: this rank holds rows
 * [rank * rows_per_rank, (rank + 1) * rows_per_rank) of W as w_shard (device
 * memory) and x in full. Every rank's buffer receives the whole y (float32,
 * nranks * rows_per_rank values) at byte offset y_offset (16-byte aligned).
 * Q4_K shards, and the Q6_K shards its tensor-core kernel takes, gather y
 * inside the matvec: each row leaves as an 8-byte {value, epoch} word for
 * every rank over NVLink, and each CTA unpacks its slice of y as the words
 * arrive, so the launch ends with the whole y on every rank (bounded wait; a
 * timeout sets the context's error word). Other types and shapes: matvec,
 * then a peer all-gather launch. Device pointers, enqueued on
 * `stream` (NULL = the context's stream), nothing allocated or synchronised.
 * Every rank must make the same calls in the same order. After SI_E_TIMEOUT
 * the buffer's exchange state is lost: destroy it and create a new one. */
int si_sharded_qmatvec_dev(si_ctx* ctx, si_peer_buffer* buf, uint32_t ggml_type, const void* w_shard,
                           uint64_t rows_per_rank, uint64_t cols, const float* x, uint64_t y_offset, void* stream);
/* Wait for the context's stream and report device errors (timed-out waits)
 * of the `_dev` calls enqueued before (commit + wait of the reference's
 * command buffers, metal.rs:2330-2335). */
int si_ctx_synchronize(si_ctx* ctx);

/* ---- greedy argmax (runtime.rs:4301-4309) -------------------------------- */
/* Largest finite value under f32::total_cmp; the last index among equals. */
int si_argmax(si_ctx* ctx, const float* logits, uint64_t n, uint32_t* index);

/* ---- synthetic Qwen3.6-shaped model ------------------------------------- */
/* Tensor ids of one decoder layer (qwen35_runtime.rs:419-446, 640-657) and of
 * the globals (stored under layer index == layers). */
enum {
  SI_T_ATTN_NORM = 0, SI_T_POST_NORM, SI_T_FFN_GATE, SI_T_FFN_UP, SI_T_FFN_DOWN,
  SI_T_SSM_QKV, SI_T_SSM_Z, SI_T_SSM_ALPHA, SI_T_SSM_BETA, SI_T_SSM_CONV, SI_T_SSM_A,
  SI_T_SSM_DT, SI_T_SSM_NORM, SI_T_SSM_OUT,
  SI_T_ATTN_Q, SI_T_ATTN_K, SI_T_ATTN_V, SI_T_ATTN_O, SI_T_ATTN_QNORM, SI_T_ATTN_KNORM,
  SI_T_TOKEN_EMBD, SI_T_OUTPUT_NORM, SI_T_OUTPUT,
  SI_T_COUNT
};

/* GgufQwen35Config (model.rs:321-442) restricted to what decode needs. */
typedef struct si_model_config {
  uint32_t hidden, intermediate, layers, vocab;
  uint32_t attn_interval;                       /* full attention where (l+1)%interval==0 */
  uint32_t attn_q_heads, attn_kv_heads, attn_head_dim, rotary_dim;
  float rope_theta;
  uint32_t gdn_key_heads, gdn_value_heads, gdn_head_dim, conv_kernel;
  float rms_eps;
  uint32_t kv_capacity;                         /* KV positions per attention layer */
  uint32_t eos_token;                           /* 0xFFFFFFFF = none */
  uint32_t mlp_type, down_type, head_type;      /* ggml types of gate/up, down, output */
  uint32_t weight_init;  /* 0: uniform quant/scale bytes (BASELINE config 1 style);
                            1: per-sub-block scale 0..8 with min ~ offset*scale and
                            dmin = d, so Q4_K/Q5_K rows are roughly zero-mean */
} si_model_config;

/* Residency / staging plan (qwen35_runtime.rs:1552-1733, planner.rs:174-251). */
typedef struct si_plan_info {
  uint64_t budget_bytes;
  uint64_t resident_weight_bytes;  /* weights uploaded once */
  uint64_t ring_bytes;             /* staging ring slots */
  uint64_t state_bytes;            /* GDN state + KV cache */
  uint64_t scratch_bytes;
  uint64_t streamed_bytes_per_token;
  uint32_t resident_layers, streamed_layers, stage_depth, head_resident;
} si_plan_info;

/* Which layers stay resident in HBM: the layer-granular forms of the
 * reference's residency selection (new_with_retained_layers_and_head,
 * qwen35_runtime.rs:1552-1733). A layer is retained when it is one of the
 * first `prefix_layers` (retained_layers), when stride != 0 and
 * layer % stride == offset % stride (retains_stride_layer, 2270-2272), or when
 * it is listed in `layers` (SI_RETAIN_FULL_LAYERS, parse_layer_set 2275-2280).
 * The output head is always resident. Without SI_RETAIN_EXACT the remaining
 * budget is filled with further leading layers, and a model that fits whole
 * stays whole; with it every other layer streams through the ring, as in the
 * reference. A retained set that the budget cannot hold beside the head, the
 * ring, state and scratch is refused with SI_E_BUDGET; a listed layer past the
 * model's depth with SI_E_INVALID.
 *
 * With SI_RETAIN_TENSORS the fields after `flags` are read too: the
 * reference's tensor-level forms, which it applies only when no layers are
 * retained by count (retained_layers == 0, qwen35_runtime.rs:1565-1640), and
 * neither are they here when prefix_layers != 0. Of every streamed layer the
 * selected tensors stay resident and only the rest goes through the ring:
 *   mlp_layers                gate and up of layers 0..mlp_layers-1
 *                             (SI_RETAIN_MLP_LAYERS, 1646-1649);
 *   mlp_stride, mlp_offset    gate and up of the stride layers
 *                             (SI_RETAIN_MLP_STRIDE / _OFFSET, 1650-1655);
 *   q6_layers                 every Q6_K tensor of layers 0..q6_layers-1
 *                             (SI_RETAIN_Q6_LAYERS, 1656-1662);
 *   down_stride, down_offset  ffn_down of the stride layers
 *                             (SI_RETAIN_DOWN_STRIDE / _OFFSET, 1667-1671);
 *   attention_stride, _offset q, k, v and output projections of the stride
 *                             layers that are full-attention layers
 *                             (SI_RETAIN_ATTENTION_STRIDE / _OFFSET, 1672-1682).
 * A stride of 0 selects nothing. The selected tensors count against the
 * budget like retained layers (SI_E_BUDGET when they do not fit). */
typedef struct si_retention {
  uint32_t prefix_layers;
  uint32_t stride, offset;
  const uint32_t* layers; /* may be NULL when n_layers is 0 */
  uint32_t n_layers;
  uint32_t flags;         /* SI_RETAIN_* */
  /* read only with SI_RETAIN_TENSORS */
  uint32_t mlp_layers, mlp_stride, mlp_offset;
  uint32_t q6_layers;
  uint32_t down_stride, down_offset;
  uint32_t attention_stride, attention_offset;
} si_retention;
#define SI_RETAIN_EXACT 1u
#define SI_RETAIN_TENSORS 2u
/* The policy for models created on `ctx` afterwards; NULL restores the
 * default (the budget-filled prefix). */
int si_ctx_set_retention(si_ctx* ctx, const si_retention* r);

/* Fill a config with the BASELINE 27B shape (hidden 5120, 64 layers, ...). */
void si_model_config_qwen36_27b(si_model_config* c);
/* Build a model with seeded synthetic weights in pinned host memory, plan
 * residency within ctx's HBM budget, upload the resident set. With a
 * communicator attached (si_ctx_comm_init) every rank builds only its shard. */
int si_model_create_synthetic(si_ctx* ctx, const si_model_config* c, uint64_t seed,
                              si_model** out);
/* A model from a qwen35 GGUF file (Qwen35Runtime over GgufModelStore,
 * qwen35_runtime.rs:1519-1750; model.rs:628-790): config from the metadata,
 * every layer's tensors checked for kind, type, shape and payload size before
 * any allocation, each rank's row shards read from the file into pinned host
 * memory, then the same residency plan and decode path as the synthetic
 * model. Projections may be Q4_K/Q5_K/Q6_K per tensor; token_embd must be
 * Q4_K; norms, conv, alpha/beta, ssm_a and ssm_dt must be F32. kv_capacity 0
 * picks min(context_length, 4096). */
int si_model_create_gguf(si_ctx* ctx, const char* path, uint32_t kv_capacity, si_model** out);
void si_model_destroy(si_model* m);
int si_model_plan(const si_model* m, si_plan_info* out);
/* The same residency plan without a device or any allocation (planner dry
 * run, plan_sequential_layers' budget check, planner.rs:174-251). */
int si_model_plan_dry(const si_model_config* c, int nranks, int rank, uint64_t budget,
                      uint32_t stage_depth, si_plan_info* out);
/* The dry run under a retention policy (NULL: the default). resident, when
 * not NULL, receives c->layers flags: 1 for a resident layer, 0 for a
 * streamed one. */
int si_model_plan_dry_retained(const si_model_config* c, int nranks, int rank, uint64_t budget,
                               uint32_t stage_depth, const si_retention* r, si_plan_info* out,
                               uint8_t* resident);
/* Which layers of a created model are resident (layers flags, as above). */
int si_model_resident_layers(const si_model* m, uint8_t* resident, uint32_t layers);
/* Bytes of each layer that stay resident while the rest of the layer streams
 * (the tensor-level retention above; 0 for whole-resident and plainly
 * streamed layers): `layers` u64 values. */
int si_model_resident_part_bytes(const si_model* m, uint64_t* part_bytes, uint32_t layers);
/* Full-tensor row ranges [begin, end) that rank `rank` of `nranks` holds of a
 * tensor (ranges: 2*max_ranges u64). No device needed. */
int si_model_shard_rows(const si_model_config* c, int nranks, int rank, uint32_t layer,
                        uint32_t tensor, uint64_t* ranges, uint32_t max_ranges,
                        uint32_t* n_ranges);
/* This rank's pinned host copy of one tensor (its shard; with one rank, the
 * full tensor). */
int si_model_host_tensor(const si_model* m, uint32_t layer, uint32_t tensor, const void** ptr,
                         uint64_t* bytes, uint32_t* ggml_type);
int si_model_reset(si_model* m);                     /* Qwen35Runtime::reset */
/* snapshot_states / restore_states (qwen35_runtime.rs:1764-1775): a device
 * copy of every layer's recurrent, conv and KV state with the token counts,
 * for rolling a speculative window back (si-qwen35-spec-probe.rs:155-169).
 * Restoring into a model of another layout or context is refused with
 * SI_E_INVALID. Free a snapshot before its context. */
typedef struct si_model_snapshot si_model_snapshot;
int si_model_snapshot_states(si_model* m, si_model_snapshot** out);
int si_model_restore_states(si_model* m, const si_model_snapshot* s);
void si_model_snapshot_free(si_model_snapshot* s);
/* embed_token (qwen35_runtime.rs:2122). */
int si_model_embed(si_model* m, uint32_t token, float* hidden_out);
/* decode_hidden (qwen35_runtime.rs:1776): hidden is read and overwritten. */
int si_model_decode_hidden(si_model* m, uint64_t position, float* hidden);
/* logits (qwen35_runtime.rs:2132). */
int si_model_logits(si_model* m, const float* hidden, float* logits);
/* decode_token (qwen35_runtime.rs:2229): embed, decode, logits, argmax. */
int si_model_decode_token(si_model* m, uint32_t token, uint64_t position, uint32_t* next,
                          float* logits /* may be NULL */);
/* run_gguf_generation (runtime.rs:3560): token-by-token prefill, greedy loop.
 * Writes up to max_new ids; *n_out receives the count (stops after EOS). */
int si_model_generate(si_model* m, const uint32_t* prompt, uint64_t n_prompt, uint64_t max_new,
                      uint32_t* out_ids, uint64_t* n_out);

/* ---- GGUF container (host only; model.rs:583-1236) ------------------------ */
/* An open GGUF v2/v3 file: metadata and tensor index parsed, payloads left on
 * disk and read on demand with pread. Errors: si_global_last_error(), with
 * the reference's messages (model.rs:1034-1120 parse_gguf). */
typedef struct si_gguf si_gguf;
/* GgufModelStore::open (model.rs:628-666). */
int si_gguf_open(const char* path, si_gguf** out);
void si_gguf_close(si_gguf* g);
int si_gguf_info(const si_gguf* g, uint32_t* version, uint64_t* tensor_count,
                 uint64_t* metadata_count);
/* Entry `index` of the tensor index in file order (GgufTensorInfo,
 * model.rs:498-505): name (owned by g; a C string, so it ends at an embedded NUL), rank, dims (the first 4, 1-padded), ggml
 * type, and the resolved payload range [data_start, data_start+data_len) that
 * runs to the next tensor's offset or to the end of the file. */
int si_gguf_tensor_info(const si_gguf* g, uint64_t index, const char** name, uint32_t* ndim,
                        uint64_t* dims, uint32_t* ggml_type, uint64_t* data_start,
                        uint64_t* data_len);
/* GgufModelStore::tensor lookup by name (model.rs:668-686). */
int si_gguf_find_tensor(const si_gguf* g, const char* name, uint64_t* index);
/* Typed metadata: u64 accepts U8/U16/U32/U64 (required_u32, model.rs:454),
 * f64 accepts F32/F64 (required_f32, model.rs:476), string (model.rs:444),
 * array_len (required_array_len, model.rs:487). */
int si_gguf_meta_u64(const si_gguf* g, const char* key, uint64_t* out);
int si_gguf_meta_f64(const si_gguf* g, const char* key, double* out);
int si_gguf_meta_string(const si_gguf* g, const char* key, const char** out);
int si_gguf_meta_array_len(const si_gguf* g, const char* key, uint64_t* out);
/* Copy bytes [offset, offset+bytes) of tensor `index`'s payload
 * (stage_tensor_payload, model.rs:867-886). */
int si_gguf_read(const si_gguf* g, uint64_t index, uint64_t offset, void* dst, uint64_t bytes);
/* Metadata keys in byte order (the reference keeps them in a BTreeMap), and a
 * key's value summarised as si-gguf-inspect prints it (summarize,
 * src/bin/si-gguf-inspect.rs:84-101: "U32(5120)", "F32(1e-6)",
 * "string(\"qwen35\")", "array(len=N, first=[...])"). Strings are owned by g. */
int si_gguf_meta_key_at(const si_gguf* g, uint64_t index, const char** key);
int si_gguf_meta_summary(const si_gguf* g, const char* key, const char** out);
/* qwen35_layer_kind (model.rs:748-783): ssm_a present = Gated DeltaNet,
 * attn_q.weight present = full attention; exactly one, and agreeing with the
 * full-attention interval. */
#define SI_LAYER_GATED_DELTA_NET 0u
#define SI_LAYER_FULL_ATTENTION 1u
int si_gguf_qwen35_layer_kind(const si_gguf* g, uint32_t layer, uint32_t* kind);
/* GgufTensorInfo::element_count / expected_payload_bytes (model.rs:512-573):
 * *known = 0 for types other than F32, F16, BF16 and the K-quants. */
int si_gguf_tensor_payload(const si_gguf* g, uint64_t index, uint64_t* elements, uint64_t* expected_bytes,
                           uint32_t* known);
/* GgufModelStore::stage_qwen35_layer_packed (model.rs:920-985): the tensors
 * of blk.<layer>. other than F32 ones and those named in `excluded`, ordered
 * by file offset and read as runs (a tensor that starts within 4096 bytes of
 * the current run's end extends it; the bytes between are read too), packed
 * back to back. The ranges, in name order, locate each tensor in the packed
 * bytes; the pair feeds si_staged_layer_upload / _bind_host directly. */
typedef struct si_gguf_packed si_gguf_packed;
int si_gguf_stage_layer_packed(const si_gguf* g, uint32_t layer, const char* const* excluded, uint32_t n_excluded,
                               si_gguf_packed** out);
int si_gguf_packed_info(const si_gguf_packed* p, const void** bytes, uint64_t* nbytes, uint32_t* n_ranges);
int si_gguf_packed_range(const si_gguf_packed* p, uint32_t i, const char** name, uint64_t* start, uint64_t* end);
void si_gguf_packed_free(si_gguf_packed* p);
/* GgufModelStore::advise_qwen35_layer (model.rs:986-1024): ask the kernel to
 * read ahead every tensor of blk.<layer>. (posix_fadvise WILLNEED over
 * page-aligned payload ranges; a hint that moves no bytes). *advised = the
 * page-aligned bytes named, as the reference returns. */
int si_gguf_advise_layer(const si_gguf* g, uint32_t layer, uint64_t* advised);
/* GgufModelStore::dequantize_q4_k / _q5_k / _q6_k (model.rs:792-850): the
 * whole tensor `index`, which must be of `ggml_type`, dequantised
 * (bit-exact); out_len = its element count. The reference's messages for a
 * type mismatch and a short payload. */
int si_gguf_dequantize_tensor(si_ctx* ctx, const si_gguf* g, uint64_t index, uint32_t ggml_type, float* out,
                              uint64_t out_len);
/* gguf_quant_matvec_many_tensors (metal.rs:4532-4638): n K-quant tensors of
 * an open GGUF file that share x (x_len must equal their column count), with
 * the reference's checks: same columns, rank 2, a K-quant type, a payload that
 * covers rows x cols. Each payload is read from the file for the call. */
int si_gguf_quant_matvec_many_tensors(si_ctx* ctx, const si_gguf* g, uint32_t n, const uint64_t* indices,
                                      const float* x, uint64_t x_len, float* const* ys);
/* gguf_matvec_tensor_rows (metal.rs:5003-5015): rows [row_start,
 * row_start+row_count) of tensor `index` (F32 or a K-quant), read from the
 * file, times x (dims[0] columns). */
int si_gguf_matvec_tensor_rows(si_ctx* ctx, const si_gguf* g, uint64_t index, uint64_t row_start,
                               uint64_t row_count, const float* x, float* y);
/* q4_k_embedding_tensor (metal.rs:3785-3811): row `token` of a rank-2 Q4_K
 * tensor, read from the file and dequantised (bit-exact). */
int si_gguf_q4_k_embedding(si_ctx* ctx, const si_gguf* g, uint64_t index, uint64_t token, float* out);
/* detect_model_format (model.rs:42-78) without loading any payload: a
 * directory whose manifest.json says format "safetensors" and dtype
 * "bfloat16", or a file starting with the GGUF magic. */
#define SI_FORMAT_SAFETENSORS 1u
#define SI_FORMAT_GGUF 2u
int si_detect_model_format(const char* path, uint32_t* format);
/* GgufQwen35Config::from_metadata (model.rs:350-417) plus the rotary width
 * (qwen35_runtime.rs:811-813) into a decode config; the ggml types of
 * blk.0.ffn_gate / blk.0.ffn_down / output fill mlp/down/head_type.
 * kv_capacity 0 picks min(context_length, 4096). */
int si_gguf_qwen35_config(const si_gguf* g, uint32_t kv_capacity, si_model_config* out);

/* ---- batched verifier (unsharded models) ---------------------------------- */
/* decode_tokens_many (qwen35_runtime.rs:2048-2120): embed n <= 8 candidate
 * tokens and run every layer over the window with one traversal of each
 * weight matrix (qwen35_decoder_block_many, 879-1289); candidate k sees the
 * GDN and KV state left by candidates < k, as sequential decode would, and
 * all n are committed to the state. hidden_out (may be NULL): n x hidden f32.
 * The final hidden states also stay on the device for si_model_logits_many.
 * A window that would overflow a KV cache is refused before any state
 * changes. Sharded models: SI_E_UNSUPPORTED. */
int si_model_decode_tokens_many(si_model* m, const uint32_t* tokens, const uint64_t* positions, uint32_t n,
                                float* hidden_out);
/* logits_many (qwen35_runtime.rs:2194-2227): output norm and head for n
 * hidden states (host n x hidden, or NULL: the device states of the last
 * decode_tokens_many of n tokens). logits (may be NULL): n x vocab; ids (may
 * be NULL): greedy argmax per candidate (runtime.rs:4301-4309). */
int si_model_logits_many(si_model* m, const float* hidden, uint32_t n, float* logits, uint32_t* ids);
/* decode_tokens_many then logits_many without a host round trip. */
int si_model_verify_many(si_model* m, const uint32_t* tokens, const uint64_t* positions, uint32_t n,
                         uint32_t* ids, float* logits);

/* ---- planner traces (planner.rs:10-251; SI-003 planner interface) -------- */
/* ActionKind, MemoryTier and PlannerMode of the reference (SI_TIER_HBM plays
 * the reference's Metal tier). */
enum { SI_ACT_PREFETCH = 0, SI_ACT_EXECUTE, SI_ACT_RETAIN, SI_ACT_EVICT, SI_ACT_WAIT, SI_ACT_RELEASE };
enum { SI_TIER_MAPPED_SOURCE = 0, SI_TIER_PINNED_HOST, SI_TIER_HBM, SI_TIER_CPU, SI_TIER_NVME };
enum { SI_MODE_RESIDENT = 0, SI_MODE_MMAP, SI_MODE_LAYER_STREAM, SI_MODE_SUBLAYER_STREAM, SI_MODE_OVERLAP,
       SI_MODE_HETEROGENEOUS };
typedef struct si_trace si_trace;
/* One action (PlannerAction, planner.rs:39-50); tensor_ids comma-separated.
 * Strings handed out by si_trace_action_at are owned by the trace. */
typedef struct si_trace_action {
  uint32_t kind, tier;
  const char* operation_id;
  const char* tensor_ids;
  uint64_t bytes, started_ns, ended_ns;
  const char* queue;
  const char* reason;
} si_trace_action;
typedef struct si_trace_summary_info {
  uint32_t mode, observed;                 /* observed: peaks were sampled */
  uint64_t actions;
  uint64_t planned_peak_hbm_bytes;          /* from the recorded residency */
  uint64_t observed_peak_hbm_bytes, observed_peak_rss_bytes;
  uint64_t resident_hbm_tensors, resident_hbm_bytes;  /* at the end of the trace */
} si_trace_summary_info;
si_trace* si_trace_create(uint32_t mode);
void si_trace_destroy(si_trace* t);
/* PlannerTrace::record (planner.rs:96-155): rejects an action that names no
 * tensor, ends before it starts, executes a non-resident tensor or evicts one
 * that is not resident; prefetch/retain in HBM update the planned peak. */
int si_trace_record(si_trace* t, const si_trace_action* action);
int si_trace_count(const si_trace* t, uint64_t* n);
int si_trace_action_at(const si_trace* t, uint64_t index, si_trace_action* out);
int si_trace_summary(const si_trace* t, si_trace_summary_info* out);
/* plan_sequential_layers (planner.rs:174-251): prefetch, execute, evict per
 * layer; tensor ids and bytes are the layers' tensors in order. */
int si_plan_sequential_layers(uint32_t layers, const char* const* operation_ids, const uint32_t* tensor_counts,
                              const char* const* tensor_ids, const uint64_t* tensor_bytes, uint64_t budget_bytes,
                              si_trace** out);
/* The model's real trace (the scheduler the reference's planner anticipates,
 * planner.rs:1-5): between begin and end, every ring copy (prefetch), layer
 * and head execution and slot reuse (evict) is recorded with CUDA event
 * timestamps on its stream; resident and already staged layers are retained.
 * trace_end synchronises, replays the actions in time order through
 * si_trace_record and checks the SI-003 invariants on the measured times: no
 * execution starts before its prefetch has landed, and no layer is evicted
 * (its slot overwritten) before its execution ends. Observed peaks are the
 * context's device peak and the process RSS. */
int si_model_trace_begin(si_model* m);
int si_model_trace_end(si_model* m, si_trace** out);

/* ---- multi-GPU row sharding over NCCL ----------------------------------- */
#define SI_COMM_ID_BYTES 128
int si_comm_unique_id(void* id_out /* SI_COMM_ID_BYTES */);
int si_ctx_comm_init(si_ctx* ctx, int nranks, int rank, const void* id);
int si_ctx_comm_info(const si_ctx* ctx, int* nranks, int* rank);

#ifdef __cplusplus
}
#endif
#endif /* SI_CUDA_H */
