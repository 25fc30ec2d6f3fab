// C ABI: context, weights and the host-memory operator entry points that
// mirror MetalContext (src/metal.rs) of the reference. Validation order and
// messages follow the reference methods so Rust callers see the same errors.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "comm.h"
#include "ctx.h"
#include "fault.h"
#include "gguf.h"
#include "kernels.cuh"
#include "qmatvec.cuh"

namespace {
thread_local std::string g_last_error;
}

struct si_weight {
  si_ctx* ctx = nullptr;
  void* dev = nullptr;         // device copy (upload) or nullptr (host-bound)
  const void* host = nullptr;  // host-bound bytes
  uint64_t bytes = 0;
  uint32_t type = 0;
  bool registered = false;
  bool view = false;  // a view into a staged layer: the layer owns the memory
};

// A packed decoder layer promoted to device memory or bound in host memory
// (PrivateStagedQwenLayer, metal.rs:1852-1869).
struct si_staged_layer {
  si_ctx* ctx = nullptr;
  uint8_t* dev = nullptr;      // upload: each range at its own 256-byte aligned offset
  const uint8_t* host = nullptr;  // bind: the caller's packed bytes
  bool registered = false;
  uint64_t bytes = 0, dev_bytes = 0;
  struct Range {
    uint64_t start, end, dev_off;
  };
  std::map<std::string, Range> ranges;
};

namespace si {

// Armed sites count down the calls still to pass; -1 = disarmed.
std::atomic<int64_t> g_fault[SI_FAULT_SITES] = {{-1}, {-1}, {-1}, {-1}};

bool fault_fire(uint32_t site) {
  if (site == 0 || site >= SI_FAULT_SITES) return false;
  int64_t v = g_fault[site].load(std::memory_order_relaxed);
  while (v >= 0)
    if (g_fault[site].compare_exchange_weak(v, v - 1)) return v == 0;
  return false;
}

int fail(si_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->err = msg;
  g_last_error = msg;
  return code;
}

int cuda_fail(si_ctx* ctx, cudaError_t e, const char* what) {
  return fail(ctx, e == cudaErrorMemoryAllocation ? SI_E_NOMEM : SI_E_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

void note_alloc(si_ctx* ctx, int64_t delta) {
  uint64_t now = ctx->allocated.fetch_add(uint64_t(delta)) + uint64_t(delta);
  uint64_t peak = ctx->peak_allocated.load();
  while (now > peak && !ctx->peak_allocated.compare_exchange_weak(peak, now)) {
  }
}

// An enqueue that returns without waiting (the `_dev` entry points): the
// reference's record_async_submission (metal.rs:1891-1947) counts it as a
// submission and as an async one.
void note_async_submission(si_ctx* ctx) {
  ctx->submitted++;
  ctx->async_submitted++;
}

static_assert(sizeof(si_ctx::qs_stream) / sizeof(cudaStream_t) == kQmvScratchSlots, "one stream per slot");

void qscratch_for(si_ctx* ctx, cudaStream_t stream, void** p, uint64_t* bytes) {
  *p = nullptr;
  *bytes = 0;
  if (!ctx->qscratch.p) return;
  if (!stream) stream = ctx->stream;
  std::lock_guard<std::mutex> lk(ctx->qs_mu);
  ctx->qs_stream[0] = ctx->stream;
  for (int i = 0; i < kQmvScratchSlots; ++i) {
    if (ctx->qs_stream[i] == stream || !ctx->qs_stream[i]) {
      ctx->qs_stream[i] = stream;
      *p = static_cast<uint8_t*>(ctx->qscratch.p) + uint64_t(i) * kQmvScratchBytes;
      *bytes = kQmvScratchBytes;
      return;
    }
  }
}

void note_weights(si_ctx* ctx, int64_t delta) {
  uint64_t now = ctx->weights.fetch_add(uint64_t(delta)) + uint64_t(delta);
  uint64_t peak = ctx->peak_weights.load();
  while (now > peak && !ctx->peak_weights.compare_exchange_weak(peak, now)) {
  }
}

int sync_and_check(si_ctx* ctx, const char* what) {
  auto t0 = std::chrono::steady_clock::now();
  ctx->submitted++;
  // the error word travels with the results: one synchronisation per call
  cudaError_t e = cudaMemcpyAsync(ctx->h_err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  ctx->waited++;
  ctx->wait_nanos += uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                  std::chrono::steady_clock::now() - t0)
                                  .count());
  if (e == cudaSuccess)
    for (const auto& pc : ctx->pending) std::memcpy(pc.dst, ctx->h_stage + pc.off, pc.bytes);
  ctx->pending.clear();
  ctx->h_stage_used = 0;
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  const int bits = *ctx->h_err;
  if (bits) {
    cudaMemset(ctx->d_err, 0, sizeof(int));
    // a kernel that gave up may have left split-group counters behind
    if (ctx->qscratch.p) cudaMemset(ctx->qscratch.p, 0, ctx->qscratch.cap);
    *ctx->h_err = 0;
    return fail(ctx, bits & (KERR_TIMEOUT_FULL | KERR_TIMEOUT_EMPTY | KERR_TIMEOUT_DRAIN)
                         ? SI_E_TIMEOUT
                         : SI_E_CUDA,
                std::string(what) + ": device error bits " + std::to_string(bits));
  }
  return SI_OK;
}

// Copy host bytes into a staging buffer on the compute stream.
static int h2d(si_ctx* ctx, DevBuf& b, const void* src, size_t bytes, const char* what) {
  if (!b.ensure(bytes)) return fail(ctx, SI_E_NOMEM, std::string(what) + ": device allocation failed");
  if (bytes) {
    cudaError_t e = cudaMemcpyAsync(b.p, src, bytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  }
  return SI_OK;
}

// Device -> caller memory, completed by the next sync_and_check: through the
// pinned staging buffer when it has room (grown while nothing is pending),
// else directly.
static int d2h(si_ctx* ctx, void* dst, const void* src, size_t bytes, const char* what) {
  if (bytes == 0) return SI_OK;
  const size_t need = (ctx->h_stage_used + bytes + 255) & ~size_t(255);
  if (need > ctx->h_stage_cap && ctx->pending.empty()) {
    if (ctx->h_stage) cudaFreeHost(ctx->h_stage);
    ctx->h_stage = nullptr;
    ctx->h_stage_cap = 0;
    const size_t cap = std::max(need, size_t(1) << 20);
    if (cudaHostAlloc(reinterpret_cast<void**>(&ctx->h_stage), cap, cudaHostAllocDefault) == cudaSuccess)
      ctx->h_stage_cap = cap;
    else
      ctx->h_stage = nullptr;
  }
  cudaError_t e;
  if (ctx->h_stage && need <= ctx->h_stage_cap) {
    e = cudaMemcpyAsync(ctx->h_stage + ctx->h_stage_used, src, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) ctx->pending.push_back({dst, ctx->h_stage_used, bytes});
    ctx->h_stage_used = need;
  } else {
    e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream);
  }
  if (e != cudaSuccess) {
    ctx->pending.clear();  // the call fails: none of its readbacks is delivered
    ctx->h_stage_used = 0;
    return cuda_fail(ctx, e, what);
  }
  return SI_OK;
}

static const char* type_label(uint32_t t) {
  return t == SI_GGML_TYPE_Q4_K ? "Q4_K" : t == SI_GGML_TYPE_Q5_K ? "Q5_K" : t == SI_GGML_TYPE_Q6_K ? "Q6_K" : "?";
}

// Shared validation of quant_k_matvec_dispatch (metal.rs:3847-3858).
static int check_qmv(si_ctx* ctx, uint32_t type, uint64_t nbytes, uint64_t rows, uint64_t cols,
                     const char* extra = "") {
  const uint32_t bb = block_bytes_of(type);
  if (bb == 0) return fail(ctx, SI_E_UNSUPPORTED, "unsupported quantized weight type");
  const std::string label = type_label(type);
  if (rows == 0 || cols == 0 || cols % 256)
    return fail(ctx, SI_E_INVALID, label + extra + " matvec dimensions are invalid");
  if (rows > 0xffffffffull || cols > kQmvMaxCols)
    return fail(ctx, SI_E_UNSUPPORTED, label + " matvec dimensions exceed backend limits");
  if (nbytes != rows * (cols / 256) * bb)
    return fail(ctx, SI_E_INVALID, label + extra + " matvec byte length is invalid");
  return SI_OK;
}

}  // namespace si

using namespace si;

extern "C" {

const char* si_global_last_error(void) { return g_last_error.c_str(); }

const char* si_last_error(const si_ctx* ctx) { return ctx ? ctx->err.c_str() : g_last_error.c_str(); }

int si_ctx_create(int device, const si_ctx_config* cfg, si_ctx** out) {
  if (!out) return fail(nullptr, SI_E_INVALID, "null output handle");
  *out = nullptr;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaSetDevice");
  int major = 0, minor = 0, sms = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (major != 10)
    return fail(nullptr, SI_E_UNSUPPORTED,
                "this backend is built for sm_100a (B200); device has compute capability " +
                    std::to_string(major) + "." + std::to_string(minor));
  auto* c = new si_ctx();
  c->device = device;
  c->sm_count = sms;
  if (cfg) c->cfg = *cfg;
  if (c->cfg.stage_depth == 0) c->cfg.stage_depth = 3;
  if (c->cfg.stage_depth > 4) c->cfg.stage_depth = 4;
  if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaMalloc(&c->d_err, 64)) != cudaSuccess ||
      (e = cudaHostAlloc(reinterpret_cast<void**>(&c->h_err), 64, cudaHostAllocDefault)) != cudaSuccess ||
      (e = cudaMalloc(&c->d_argmax, 64)) != cudaSuccess ||
      (e = cudaMalloc(&c->d_index, 64)) != cudaSuccess) {
    int rc = cuda_fail(nullptr, e, "context creation");
    si_ctx_destroy(c);
    return rc;
  }
  if (!c->qscratch.ensure(kQmvScratchBytes * kQmvScratchSlots) || cudaMemset(c->qscratch.p, 0, c->qscratch.cap) != cudaSuccess) {
    int rc = fail(nullptr, SI_E_NOMEM, "context creation: matvec scratch allocation failed");
    si_ctx_destroy(c);
    return rc;
  }
  cudaMemset(c->d_err, 0, 64);
  cudaMemset(c->d_argmax, 0, 64);
  cudaDeviceSynchronize();
  *out = c;
  return SI_OK;
}

void si_ctx_destroy(si_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  comm_destroy(ctx);
  for (auto& b : ctx->in) b.release();
  for (auto& b : ctx->out) b.release();
  for (auto& b : ctx->wbuf) b.release();
  ctx->scratch.release();
  ctx->qscratch.release();
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->h_err) cudaFreeHost(ctx->h_err);
  if (ctx->h_stage) cudaFreeHost(ctx->h_stage);
  if (ctx->d_argmax) cudaFree(ctx->d_argmax);
  if (ctx->d_index) cudaFree(ctx->d_index);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
  delete ctx;
}

int si_device_probe(int device, si_device_info* out) {
  if (!out) return fail(nullptr, SI_E_INVALID, "invalid probe arguments");
  std::memset(out, 0, sizeof(*out));
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fail(nullptr, SI_E_CUDA, "no CUDA device found");
  }
  if (device < 0 || device >= n) return fail(nullptr, SI_E_INVALID, "device ordinal out of range");
  cudaDeviceProp p;
  if ((e = cudaGetDeviceProperties(&p, device)) != cudaSuccess) return cuda_fail(nullptr, e, "device properties");
  std::snprintf(out->name, sizeof(out->name), "%s", p.name);
  out->total_bytes = p.totalGlobalMem;
  out->sm_count = uint32_t(p.multiProcessorCount);
  out->cc_major = uint32_t(p.major);
  out->cc_minor = uint32_t(p.minor);
  out->device_count = uint32_t(n);
  return SI_OK;
}

int si_ctx_info(const si_ctx* ctx, int* device, int* sm_count) {
  if (!ctx) return SI_E_INVALID;
  if (device) *device = ctx->device;
  if (sm_count) *sm_count = ctx->sm_count;
  return SI_OK;
}

void* si_ctx_stream(si_ctx* ctx) { return ctx ? ctx->stream : nullptr; }

int si_get_stats(const si_ctx* ctx, si_stats* o) {
  if (!ctx || !o) return SI_E_INVALID;
  o->current_allocated_bytes = ctx->allocated.load();
  o->peak_allocated_bytes = ctx->peak_allocated.load();
  o->peak_active_weight_bytes = ctx->peak_weights.load();
  o->peak_kv_bytes = ctx->peak_kv.load();
  o->peak_scratch_bytes = ctx->peak_scratch.load();
  o->submitted = ctx->submitted.load();
  o->waited = ctx->waited.load();
  o->wait_nanos = ctx->wait_nanos.load();
  o->async_submitted = ctx->async_submitted.load();
  return SI_OK;
}

int si_stats_delta(const si_stats* after, const si_stats* before, si_stats* out) {
  if (!after || !before || !out) return SI_E_INVALID;
  auto sat = [](uint64_t a, uint64_t b) { return a > b ? a - b : 0; };
  *out = *after;
  out->submitted = sat(after->submitted, before->submitted);
  out->async_submitted = sat(after->async_submitted, before->async_submitted);
  out->waited = sat(after->waited, before->waited);
  out->wait_nanos = sat(after->wait_nanos, before->wait_nanos);
  return SI_OK;
}

int si_reset_peaks(si_ctx* ctx) {
  if (!ctx) return SI_E_INVALID;
  ctx->peak_allocated = ctx->allocated.load();
  ctx->peak_weights = ctx->weights.load();
  ctx->peak_kv = 0;
  ctx->peak_scratch = 0;
  return SI_OK;
}

// ---- weights ----------------------------------------------------------------
int si_weight_upload(si_ctx* ctx, const void* host, uint64_t bytes, uint32_t type,
                     si_weight** out) {
  if (!ctx || !out || (!host && bytes)) return fail(ctx, SI_E_INVALID, "invalid weight upload arguments");
  std::lock_guard<std::mutex> lk(ctx->upload_mu);
  cudaSetDevice(ctx->device);
  auto* w = new si_weight();
  w->ctx = ctx;
  w->bytes = bytes;
  w->type = type;
  cudaError_t e = fault_fire(SI_FAULT_DEVICE_ALLOC) ? cudaErrorMemoryAllocation : cudaMalloc(&w->dev, bytes + 64);
  if (e != cudaSuccess) {
    w->dev = nullptr;
    delete w;
    return cuda_fail(ctx, e, "quantized weight upload");
  }
  cudaMemset(static_cast<uint8_t*>(w->dev) + bytes, 0, 64);
  e = cudaMemcpyAsync(w->dev, host, bytes, cudaMemcpyHostToDevice, ctx->copy_stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->copy_stream);
  if (e != cudaSuccess) {
    cudaFree(w->dev);
    delete w;
    return cuda_fail(ctx, e, "quantized weight upload");
  }
  note_alloc(ctx, int64_t(bytes + 64));
  note_weights(ctx, int64_t(bytes));
  *out = w;
  return SI_OK;
}

int si_weight_bind_host(si_ctx* ctx, const void* host, uint64_t bytes, uint32_t type,
                        si_weight** out) {
  if (!ctx || !out || !host) return fail(ctx, SI_E_INVALID, "invalid weight binding arguments");
  auto* w = new si_weight();
  w->ctx = ctx;
  w->host = host;
  w->bytes = bytes;
  w->type = type;
  // Page-lock so the per-use copy runs at full PCIe/C2C speed; memory that is
  // already pinned (or cannot be registered) is used as is.
  cudaError_t e = cudaHostRegister(const_cast<void*>(host), bytes, cudaHostRegisterReadOnly);
  if (e == cudaSuccess) w->registered = true;
  else cudaGetLastError();
  *out = w;
  return SI_OK;
}

void si_weight_free(si_weight* w) {
  if (!w) return;
  if (w->view) {
    delete w;
    return;
  }
  if (w->dev) {
    cudaSetDevice(w->ctx->device);
    cudaFree(w->dev);
    note_alloc(w->ctx, -int64_t(w->bytes + 64));
    note_weights(w->ctx, -int64_t(w->bytes));
  }
  if (w->registered) cudaHostUnregister(const_cast<void*>(w->host));
  delete w;
}

uint64_t si_weight_bytes(const si_weight* w) { return w ? w->bytes : 0; }
uint32_t si_weight_type(const si_weight* w) { return w ? w->type : 0; }
const void* si_weight_device_ptr(const si_weight* w) { return w ? w->dev : nullptr; }

}  // extern "C"

namespace si {
// Device pointer of a weight for this call (host-bound weights are copied
// into staging buffer `slot`).
static int weight_dev(si_ctx* ctx, const si_weight* w, int slot, const uint8_t** out) {
  if (w->dev) {
    *out = static_cast<const uint8_t*>(w->dev);
    return SI_OK;
  }
  int rc = h2d(ctx, ctx->wbuf[slot], w->host, w->bytes, "mapped weight staging");
  if (rc) return rc;
  *out = ctx->wbuf[slot].as<uint8_t>();
  return SI_OK;
}
}  // namespace si

extern "C" {

// ---- dequant -----------------------------------------------------------------
static int dequantize_dev_impl(si_ctx* ctx, uint32_t type, const void* bytes_dev, uint64_t elements,
                      float* out_dev, void* stream) {
  if (!ctx || block_bytes_of(type) == 0) return fail(ctx, SI_E_UNSUPPORTED, "unsupported quantized type");
  if (elements == 0 || elements % 256) return fail(ctx, SI_E_INVALID, "element count must be a non-zero multiple of 256");
  launch_dequant(type, static_cast<const uint8_t*>(bytes_dev), elements, out_dev,
                 stream ? static_cast<cudaStream_t>(stream) : ctx->stream);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SI_OK : cuda_fail(ctx, e, "dequant launch");
}

int si_dequantize_dev(si_ctx* ctx, uint32_t type, const void* bytes_dev, uint64_t elements,
                      float* out_dev, void* stream) {
  const int rc = dequantize_dev_impl(ctx, type, bytes_dev, elements, out_dev, stream);
  if (rc == SI_OK) note_async_submission(ctx);
  return rc;
}

int si_dequantize(si_ctx* ctx, uint32_t type, const void* bytes, uint64_t nbytes,
                  uint64_t elements, float* out) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  const uint32_t bb = block_bytes_of(type);
  const char* label = type_label(type);
  if (bb == 0) return fail(ctx, SI_E_UNSUPPORTED, "unsupported quantized type");
  if (elements == 0 || elements % 256)
    return fail(ctx, SI_E_INVALID, std::string(label) + " element count must be a non-zero multiple of 256");
  if (nbytes != elements / 256 * bb)
    return fail(ctx, SI_E_INVALID, std::string(label) + " data has " + std::to_string(nbytes) +
                                       " bytes; expected " + std::to_string(elements / 256 * bb));
  int rc = h2d(ctx, ctx->in[0], bytes, nbytes, "dequant input");
  if (rc) return rc;
  if (!ctx->out[0].ensure(elements * 4)) return fail(ctx, SI_E_NOMEM, "dequant output allocation failed");
  launch_dequant(type, ctx->in[0].as<uint8_t>(), elements, ctx->out[0].as<float>(), ctx->stream);
  if ((rc = d2h(ctx, out, ctx->out[0].p, elements * 4, "dequant readback"))) return rc;
  return sync_and_check(ctx, "dequant command");
}

int si_q4_k_embedding_row(si_ctx* ctx, const void* row, uint64_t nbytes, uint64_t columns,
                          float* out) {
  if (!ctx) return SI_E_INVALID;
  if (columns == 0 || columns % 256) return fail(ctx, SI_E_INVALID, "Q4_K embedding dimension is invalid");
  if (nbytes != columns / 256 * 144) return fail(ctx, SI_E_INVALID, "Q4_K embedding row byte length is invalid");
  return si_dequantize(ctx, SI_GGML_TYPE_Q4_K, row, nbytes, columns, out);
}

// ---- matvec --------------------------------------------------------------------
static int qmatvec_dev_impl(si_ctx* ctx, uint32_t type, const void* w_dev, uint64_t rows, uint64_t cols,
                   const float* x_dev, float* y_dev, void* stream) {
  if (!ctx) return SI_E_INVALID;
  int rc = check_qmv(ctx, type, rows * (cols / 256) * block_bytes_of(type), rows, cols);
  if (rc) return rc;
  QmvParams p = {};
  p.type = type;
  p.cols = uint32_t(cols);
  p.nseg = 1;
  p.seg[0] = {static_cast<const uint8_t*>(w_dev), y_dev, nullptr, uint32_t(rows), 0};
  p.items = uint32_t(rows);
  p.xmode = XM_RAW;
  p.x = x_dev;
  p.err = ctx->d_err;
  qscratch_for(ctx, stream ? static_cast<cudaStream_t>(stream) : ctx->stream, &p.scratch, &p.scratch_bytes);
  std::string msg;
  // Programmatic dependent launch: back-to-back matvecs overlap the next
  // kernel's weight prefetch with this one's tail (x/y are read/written only
  // after griddepcontrol.wait).
  rc = launch_qmv(p, stream ? static_cast<cudaStream_t>(stream) : ctx->stream, ctx->sm_count,
                  true, &msg);
  return rc ? fail(ctx, rc, msg) : SI_OK;
}

int si_qmatvec_dev(si_ctx* ctx, uint32_t type, const void* w_dev, uint64_t rows, uint64_t cols,
                   const float* x_dev, float* y_dev, void* stream) {
  const int rc = qmatvec_dev_impl(ctx, type, w_dev, rows, cols, x_dev, y_dev, stream);
  if (rc == SI_OK) note_async_submission(ctx);
  return rc;
}

int si_gguf_quant_matvec_bytes(si_ctx* ctx, uint32_t type, const void* w, uint64_t nbytes,
                               uint64_t rows, uint64_t cols, const float* x, float* y) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  int rc = check_qmv(ctx, type, nbytes, rows, cols);
  if (rc) return rc;
  if ((rc = h2d(ctx, ctx->wbuf[0], w, nbytes, "matvec weight staging"))) return rc;
  if ((rc = h2d(ctx, ctx->in[0], x, cols * 4, "matvec input"))) return rc;
  if (!ctx->out[0].ensure(rows * 4)) return fail(ctx, SI_E_NOMEM, "matvec output allocation failed");
  QmvParams p = {};
  p.type = type;
  p.cols = uint32_t(cols);
  p.nseg = 1;
  p.seg[0] = {ctx->wbuf[0].as<uint8_t>(), ctx->out[0].as<float>(), nullptr, uint32_t(rows), 0};
  p.items = uint32_t(rows);
  p.x = ctx->in[0].as<float>();
  p.err = ctx->d_err;
  qscratch_for(ctx, ctx->stream, &p.scratch, &p.scratch_bytes);
  std::string msg;
  if ((rc = launch_qmv(p, ctx->stream, ctx->sm_count, false, &msg))) return fail(ctx, rc, msg);
  if ((rc = d2h(ctx, y, ctx->out[0].p, rows * 4, "matvec readback"))) return rc;
  return sync_and_check(ctx, (std::string(type_label(type)) + " matvec command").c_str());
}

int si_q4_k_matvec(si_ctx* ctx, const void* w, uint64_t nbytes, uint64_t rows, uint64_t cols,
                   const float* x, float* y) {
  return si_gguf_quant_matvec_bytes(ctx, SI_GGML_TYPE_Q4_K, w, nbytes, rows, cols, x, y);
}
int si_q5_k_matvec(si_ctx* ctx, const void* w, uint64_t nbytes, uint64_t rows, uint64_t cols,
                   const float* x, float* y) {
  return si_gguf_quant_matvec_bytes(ctx, SI_GGML_TYPE_Q5_K, w, nbytes, rows, cols, x, y);
}
int si_q6_k_matvec(si_ctx* ctx, const void* w, uint64_t nbytes, uint64_t rows, uint64_t cols,
                   const float* x, float* y) {
  return si_gguf_quant_matvec_bytes(ctx, SI_GGML_TYPE_Q6_K, w, nbytes, rows, cols, x, y);
}

int si_gguf_quant_matvec_many_weights(si_ctx* ctx, uint32_t n, const si_weight* const* ws,
                                      const uint64_t* rows, const uint64_t* cols, const float* x,
                                      float* const* ys) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (n == 0 || n > 3) return fail(ctx, SI_E_INVALID, "grouped quantized matvec needs 1..3 weights");
  const uint32_t type = ws[0]->type;
  uint64_t total = 0;
  for (uint32_t i = 0; i < n; ++i) {
    if (ws[i]->type != type || cols[i] != cols[0])
      return fail(ctx, SI_E_INVALID, "grouped quantized matvec weights must share type and columns");
    int rc = check_qmv(ctx, type, ws[i]->bytes, rows[i], cols[i], " retained");
    if (rc) return rc;
    total += rows[i];
  }
  int rc = h2d(ctx, ctx->in[0], x, cols[0] * 4, "grouped matvec input");
  if (rc) return rc;
  if (!ctx->out[0].ensure(total * 4)) return fail(ctx, SI_E_NOMEM, "grouped matvec output allocation failed");
  QmvParams p = {};
  p.type = type;
  p.cols = uint32_t(cols[0]);
  p.nseg = n;
  uint64_t off = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const uint8_t* wd;
    if ((rc = weight_dev(ctx, ws[i], int(i), &wd))) return rc;
    p.seg[i] = {wd, ctx->out[0].as<float>() + off, nullptr, uint32_t(rows[i]), 0};
    off += rows[i];
  }
  p.items = uint32_t(total);
  p.x = ctx->in[0].as<float>();
  p.err = ctx->d_err;
  qscratch_for(ctx, ctx->stream, &p.scratch, &p.scratch_bytes);
  std::string msg;
  if ((rc = launch_qmv(p, ctx->stream, ctx->sm_count, false, &msg))) return fail(ctx, rc, msg);
  off = 0;
  for (uint32_t i = 0; i < n; ++i) {
    if ((rc = d2h(ctx, ys[i], ctx->out[0].as<float>() + off, rows[i] * 4, "grouped readback"))) return rc;
    off += rows[i];
  }
  return sync_and_check(ctx, "grouped matvec command");
}

int si_gguf_quant_matvec_weight(si_ctx* ctx, const si_weight* w, uint64_t rows, uint64_t cols,
                                const float* x, float* y) {
  if (!ctx || !w) return fail(ctx, SI_E_INVALID, "null weight");
  if (block_bytes_of(w->type) == 0) return fail(ctx, SI_E_UNSUPPORTED, "unsupported retained quantized weight type");
  uint64_t r = rows, c = cols;
  float* yy = y;
  return si_gguf_quant_matvec_many_weights(ctx, 1, &w, &r, &c, x, &yy);
}

// Batched matvec over host or retained weights (metal.rs:4067-4230): inputs
// [batch][cols], outputs [batch][rows].
static int qmm_host(si_ctx* ctx, uint32_t type, const uint8_t* w_dev, uint64_t rows, uint64_t cols,
                    uint64_t batch, const float* inputs, float* outputs) {
  int rc = h2d(ctx, ctx->in[0], inputs, batch * cols * 4, "batched matvec input");
  if (rc) return rc;
  if (!ctx->out[0].ensure(batch * rows * 4)) return fail(ctx, SI_E_NOMEM, "batched matvec output allocation failed");
  QmmParams p = {};
  p.type = type;
  p.rows = uint32_t(rows);
  p.cols = uint32_t(cols);
  p.batch = uint32_t(batch);
  p.w = w_dev;
  p.x = ctx->in[0].as<float>();
  p.ldx = cols;
  p.y = ctx->out[0].as<float>();
  p.ldy = rows;
  p.err = ctx->d_err;
  qscratch_for(ctx, ctx->stream, &p.qscratch, &p.qscratch_bytes);
  const uint64_t need = qmm_tc_scratch_bytes(uint32_t(rows), uint32_t(cols), uint32_t(batch), ctx->sm_count);
  if (ctx->scratch.ensure(need)) {
    p.scratch = ctx->scratch.p;
    p.scratch_bytes = need;
  }
  std::string msg;
  if ((rc = launch_qmm(p, ctx->stream, ctx->sm_count, false, &msg))) return fail(ctx, rc, msg);
  if ((rc = d2h(ctx, outputs, ctx->out[0].p, batch * rows * 4, "batched matvec readback"))) return rc;
  return sync_and_check(ctx, "batched quantized matvec command");
}

int si_gguf_quant_matmul_many_bytes(si_ctx* ctx, uint32_t type, const void* w, uint64_t nbytes, uint64_t rows,
                                    uint64_t cols, uint64_t batch, const float* inputs, float* outputs) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (batch == 0 || batch > kQmmMaxBatch || rows == 0 || cols == 0 || cols % 256 || rows > 0xffffffffull ||
      cols > kQmvMaxCols)
    return fail(ctx, SI_E_INVALID, "batched quantized matvec dimensions are invalid");
  if (!inputs || !outputs || !w) return fail(ctx, SI_E_INVALID, "batched quantized input length is invalid");
  const uint32_t bb = block_bytes_of(type);
  if (bb == 0) return fail(ctx, SI_E_UNSUPPORTED, "unsupported batched quantized weight type");
  if (nbytes != rows * (cols / 256) * bb) return fail(ctx, SI_E_INVALID, "batched quantized weight byte length is invalid");
  int rc = h2d(ctx, ctx->wbuf[0], w, nbytes, "batched matvec weight staging");
  if (rc) return rc;
  return qmm_host(ctx, type, ctx->wbuf[0].as<uint8_t>(), rows, cols, batch, inputs, outputs);
}

int si_gguf_quant_matmul_many_weight(si_ctx* ctx, const si_weight* w, uint64_t rows, uint64_t cols, uint64_t batch,
                                     const float* inputs, float* outputs) {
  if (!ctx || !w) return fail(ctx, SI_E_INVALID, "null weight");
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (batch == 0 || batch > kQmmMaxBatch || rows == 0 || cols == 0 || cols % 256 || rows > 0xffffffffull ||
      cols > kQmvMaxCols)
    return fail(ctx, SI_E_INVALID, "batched retained quantized dimensions are invalid");
  if (!inputs || !outputs) return fail(ctx, SI_E_INVALID, "batched retained quantized input length is invalid");
  const uint32_t bb = block_bytes_of(w->type);
  if (bb == 0) return fail(ctx, SI_E_UNSUPPORTED, "unsupported retained batched quantized type");
  if (w->bytes != rows * (cols / 256) * bb) return fail(ctx, SI_E_INVALID, "retained batched weight byte length is invalid");
  const uint8_t* wd;
  int rc = weight_dev(ctx, w, 0, &wd);
  if (rc) return rc;
  return qmm_host(ctx, w->type, wd, rows, cols, batch, inputs, outputs);
}

static int qmatmul_many_dev_impl(si_ctx* ctx, uint32_t type, const void* w_dev, uint64_t rows, uint64_t cols, uint64_t batch,
                        const float* x_dev, float* y_dev, void* stream) {
  if (!ctx) return SI_E_INVALID;
  if (batch == 0 || batch > kQmmMaxBatch || rows == 0 || cols == 0 || cols % 256 || rows > 0xffffffffull)
    return fail(ctx, SI_E_INVALID, "batched quantized matvec dimensions are invalid");
  QmmParams p = {};
  p.type = type;
  p.rows = uint32_t(rows);
  p.cols = uint32_t(cols);
  p.batch = uint32_t(batch);
  p.w = static_cast<const uint8_t*>(w_dev);
  p.x = x_dev;
  p.ldx = cols;
  p.y = y_dev;
  p.ldy = rows;
  p.err = ctx->d_err;
  qscratch_for(ctx, stream ? static_cast<cudaStream_t>(stream) : ctx->stream, &p.qscratch, &p.qscratch_bytes);
  // the tensor-core form's scratch is the context's (calls on one context
  // are serialised on the host, and kernels on one stream in order)
  const uint64_t need = qmm_tc_scratch_bytes(uint32_t(rows), uint32_t(cols), uint32_t(batch), ctx->sm_count);
  {
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (ctx->scratch.ensure(need)) {
      p.scratch = ctx->scratch.p;
      p.scratch_bytes = need;
    }
  }
  std::string msg;
  int rc = launch_qmm(p, stream ? static_cast<cudaStream_t>(stream) : ctx->stream, ctx->sm_count, true, &msg);
  return rc ? fail(ctx, rc, msg) : SI_OK;
}

int si_qmatmul_many_dev(si_ctx* ctx, uint32_t type, const void* w_dev, uint64_t rows, uint64_t cols, uint64_t batch,
                        const float* x_dev, float* y_dev, void* stream) {
  const int rc = qmatmul_many_dev_impl(ctx, type, w_dev, rows, cols, batch, x_dev, y_dev, stream);
  if (rc == SI_OK) note_async_submission(ctx);
  return rc;
}

int si_f32_matvec(si_ctx* ctx, const float* w, uint64_t rows, uint64_t cols, const float* x,
                  float* y) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (rows == 0 || cols == 0) return fail(ctx, SI_E_INVALID, "F32 matvec dimensions are invalid");
  // column counts that are not a multiple of 4 are padded on upload
  const uint64_t cp = (cols + 3) / 4 * 4;
  std::vector<float> padded;
  const float* src = w;
  std::vector<float> xp;
  const float* xs = x;
  if (cp != cols) {
    padded.assign(rows * cp, 0.f);
    for (uint64_t r = 0; r < rows; ++r) std::memcpy(&padded[r * cp], w + r * cols, cols * 4);
    src = padded.data();
    xp.assign(cp, 0.f);
    std::memcpy(xp.data(), x, cols * 4);
    xs = xp.data();
  }
  int rc;
  if ((rc = h2d(ctx, ctx->wbuf[0], src, rows * cp * 4, "F32 matvec weights"))) return rc;
  if ((rc = h2d(ctx, ctx->in[0], xs, cp * 4, "F32 matvec input"))) return rc;
  if (!ctx->out[0].ensure(rows * 4)) return fail(ctx, SI_E_NOMEM, "F32 matvec output allocation failed");
  launch_f32_matvec(ctx->wbuf[0].as<float>(), rows, cp, ctx->in[0].as<float>(), ctx->out[0].as<float>(), ctx->stream);
  if ((rc = d2h(ctx, y, ctx->out[0].p, rows * 4, "F32 matvec readback"))) return rc;
  return sync_and_check(ctx, "F32 matvec command");
}

// ---- fused SwiGLU ------------------------------------------------------------
static int fused_gate_up_dev_impl(si_ctx* ctx, uint32_t type, const void* gate_dev, const void* up_dev,
                         uint64_t rows, uint64_t cols, const float* x_dev, float* out_dev,
                         void* stream) {
  if (!ctx) return SI_E_INVALID;
  int rc = check_qmv(ctx, type, rows * (cols / 256) * block_bytes_of(type), rows, cols, " fused gate/up");
  if (rc) return rc;
  QmvParams p = {};
  p.type = type;
  p.cols = uint32_t(cols);
  p.nseg = 2;
  p.pair = 1;
  p.seg[0] = {static_cast<const uint8_t*>(gate_dev), out_dev, nullptr, uint32_t(rows), 0};
  p.seg[1] = {static_cast<const uint8_t*>(up_dev), out_dev, nullptr, uint32_t(rows), 0};
  p.items = uint32_t(rows);
  p.x = x_dev;
  p.err = ctx->d_err;
  qscratch_for(ctx, stream ? static_cast<cudaStream_t>(stream) : ctx->stream, &p.scratch, &p.scratch_bytes);
  std::string msg;
  rc = launch_qmv(p, stream ? static_cast<cudaStream_t>(stream) : ctx->stream, ctx->sm_count, true, &msg);
  return rc ? fail(ctx, rc, msg) : SI_OK;
}

int si_fused_gate_up_dev(si_ctx* ctx, uint32_t type, const void* gate_dev, const void* up_dev,
                         uint64_t rows, uint64_t cols, const float* x_dev, float* out_dev,
                         void* stream) {
  const int rc = fused_gate_up_dev_impl(ctx, type, gate_dev, up_dev, rows, cols, x_dev, out_dev, stream);
  if (rc == SI_OK) note_async_submission(ctx);
  return rc;
}

static int fused_mlp_dev_impl(si_ctx* ctx, uint32_t gate_type, const void* gate_dev, const void* up_dev,
                     uint32_t down_type, const void* down_dev, uint64_t inter, uint64_t hidden,
                     const float* x_dev, float* act_dev, float* y_dev, void* stream) {
  int rc = fused_gate_up_dev_impl(ctx, gate_type, gate_dev, up_dev, inter, hidden, x_dev, act_dev, stream);
  if (rc) return rc;
  return qmatvec_dev_impl(ctx, down_type, down_dev, hidden, inter, act_dev, y_dev, stream);
}

int si_fused_mlp_dev(si_ctx* ctx, uint32_t gate_type, const void* gate_dev, const void* up_dev,
                     uint32_t down_type, const void* down_dev, uint64_t inter, uint64_t hidden,
                     const float* x_dev, float* act_dev, float* y_dev, void* stream) {
  const int rc =
      fused_mlp_dev_impl(ctx, gate_type, gate_dev, up_dev, down_type, down_dev, inter, hidden, x_dev, act_dev, y_dev, stream);
  if (rc == SI_OK) note_async_submission(ctx);
  return rc;
}

static int gate_up_impl(si_ctx* ctx, const uint8_t* g, const uint8_t* u, uint64_t rows,
                        uint64_t cols, const float* x, float* out) {
  int rc;
  if ((rc = h2d(ctx, ctx->in[0], x, cols * 4, "fused gate/up input"))) return rc;
  if (!ctx->out[0].ensure(rows * 4)) return fail(ctx, SI_E_NOMEM, "fused gate/up output allocation failed");
  if ((rc = fused_gate_up_dev_impl(ctx, SI_GGML_TYPE_Q4_K, g, u, rows, cols, ctx->in[0].as<float>(),
                                 ctx->out[0].as<float>(), ctx->stream)))
    return rc;
  if ((rc = d2h(ctx, out, ctx->out[0].p, rows * 4, "fused gate/up readback"))) return rc;
  return sync_and_check(ctx, "Q4_K fused gate/up command");
}

int si_q4_k_fused_gate_up(si_ctx* ctx, const void* gate, const void* up, uint64_t nbytes,
                          uint64_t rows, uint64_t cols, const float* x, float* out) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (rows == 0 || cols == 0 || cols % 256)
    return fail(ctx, SI_E_INVALID, "Q4_K fused gate/up dimensions are invalid");
  if (nbytes != rows * (cols / 256) * 144)
    return fail(ctx, SI_E_INVALID, "Q4_K fused gate/up byte length is invalid");
  int rc;
  if ((rc = h2d(ctx, ctx->wbuf[0], gate, nbytes, "gate staging"))) return rc;
  if ((rc = h2d(ctx, ctx->wbuf[1], up, nbytes, "up staging"))) return rc;
  return gate_up_impl(ctx, ctx->wbuf[0].as<uint8_t>(), ctx->wbuf[1].as<uint8_t>(), rows, cols, x, out);
}

int si_q4_k_fused_gate_up_weights(si_ctx* ctx, const si_weight* gate, const si_weight* up,
                                  uint64_t rows, uint64_t cols, const float* x, float* out) {
  if (!ctx || !gate || !up) return fail(ctx, SI_E_INVALID, "null weight");
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (gate->type != SI_GGML_TYPE_Q4_K || up->type != SI_GGML_TYPE_Q4_K)
    return fail(ctx, SI_E_INVALID, "Q4_K fused gate/up weights must be Q4_K");
  if (rows == 0 || cols == 0 || cols % 256)
    return fail(ctx, SI_E_INVALID, "Q4_K fused gate/up dimensions are invalid");
  const uint64_t nb = rows * (cols / 256) * 144;
  if (gate->bytes != nb || up->bytes != nb)
    return fail(ctx, SI_E_INVALID, "Q4_K fused gate/up byte length is invalid");
  const uint8_t *g, *u;
  int rc;
  if ((rc = weight_dev(ctx, gate, 0, &g)) || (rc = weight_dev(ctx, up, 1, &u))) return rc;
  return gate_up_impl(ctx, g, u, rows, cols, x, out);
}

int si_gguf_quant_fused_mlp_weights(si_ctx* ctx, const si_weight* gate, const si_weight* up,
                                    const si_weight* down, uint64_t gate_rows, uint64_t cols,
                                    uint64_t down_rows, const float* x, float* y) {
  if (!ctx || !gate || !up || !down) return fail(ctx, SI_E_INVALID, "null weight");
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (gate->type != up->type || block_bytes_of(gate->type) == 0 || block_bytes_of(down->type) == 0)
    return fail(ctx, SI_E_INVALID, "fused MLP weights have unsupported types");
  if (gate_rows == 0 || cols == 0 || cols % 256 || down_rows == 0 || gate_rows % 256)
    return fail(ctx, SI_E_INVALID, "fused MLP dimensions are invalid");
  if (gate->bytes != gate_rows * (cols / 256) * block_bytes_of(gate->type) || up->bytes != gate->bytes ||
      down->bytes != down_rows * (gate_rows / 256) * block_bytes_of(down->type))
    return fail(ctx, SI_E_INVALID, "fused MLP byte length is invalid");
  const uint8_t *g, *u, *d;
  int rc;
  if ((rc = weight_dev(ctx, gate, 0, &g)) || (rc = weight_dev(ctx, up, 1, &u)) ||
      (rc = weight_dev(ctx, down, 2, &d)))
    return rc;
  if ((rc = h2d(ctx, ctx->in[0], x, cols * 4, "fused MLP input"))) return rc;
  if (!ctx->out[0].ensure(gate_rows * 4) || !ctx->out[1].ensure(down_rows * 4))
    return fail(ctx, SI_E_NOMEM, "fused MLP output allocation failed");
  if ((rc = fused_mlp_dev_impl(ctx, gate->type, g, u, down->type, d, gate_rows, cols,
                             ctx->in[0].as<float>(), ctx->out[0].as<float>(), ctx->out[1].as<float>(),
                             ctx->stream)))
    return rc;
  if ((rc = d2h(ctx, y, ctx->out[1].p, down_rows * 4, "fused MLP readback"))) return rc;
  return sync_and_check(ctx, "fused MLP command");
}

// ---- Gated DeltaNet primitives -------------------------------------------------
int si_gated_delta_step(si_ctx* ctx, const float* q, const float* k, const float* v,
                        const float* gate, const float* beta, const float* state_in,
                        uint64_t heads, uint64_t kd, uint64_t vd, float* out, float* state_out) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (heads == 0 || kd == 0 || vd == 0 || vd > 256)  // metal.rs:3134
    return fail(ctx, SI_E_INVALID, "Gated DeltaNet dimensions are invalid");
  const uint64_t hk = heads * kd, sv = hk * vd;
  int rc;
  if ((rc = h2d(ctx, ctx->in[0], q, hk * 4, "gdn q")) || (rc = h2d(ctx, ctx->in[1], k, hk * 4, "gdn k")) ||
      (rc = h2d(ctx, ctx->in[2], v, heads * vd * 4, "gdn v")) ||
      (rc = h2d(ctx, ctx->in[3], gate, heads * 4, "gdn gate")) ||
      (rc = h2d(ctx, ctx->in[4], beta, heads * 4, "gdn beta")) ||
      (rc = h2d(ctx, ctx->in[5], state_in, sv * 4, "gdn state")))
    return rc;
  if (!ctx->out[0].ensure(heads * vd * 4)) return fail(ctx, SI_E_NOMEM, "gdn output allocation failed");
  launch_gdn_step(ctx->in[5].as<float>(), ctx->in[0].as<float>(), ctx->in[1].as<float>(),
                  ctx->in[2].as<float>(), ctx->in[3].as<float>(), ctx->in[4].as<float>(),
                  uint32_t(heads), uint32_t(kd), uint32_t(vd), ctx->out[0].as<float>(), ctx->stream);
  if ((rc = d2h(ctx, out, ctx->out[0].p, heads * vd * 4, "gdn readback")) ||
      (rc = d2h(ctx, state_out, ctx->in[5].p, sv * 4, "gdn state readback")))
    return rc;
  return sync_and_check(ctx, "Gated DeltaNet step command");
}

int si_causal_conv1d_step(si_ctx* ctx, const float* x, const float* state_in, const float* w,
                          uint64_t channels, uint64_t kernel, float* out, float* state_out) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (channels == 0 || kernel < 2) return fail(ctx, SI_E_INVALID, "causal convolution dimensions are invalid");
  const uint64_t sb = channels * (kernel - 1) * 4;
  int rc;
  if ((rc = h2d(ctx, ctx->in[0], x, channels * 4, "conv input")) ||
      (rc = h2d(ctx, ctx->in[1], state_in, sb, "conv state")) ||
      (rc = h2d(ctx, ctx->in[2], w, channels * kernel * 4, "conv weights")))
    return rc;
  if (!ctx->out[0].ensure(channels * 4) || !ctx->out[1].ensure(sb))
    return fail(ctx, SI_E_NOMEM, "conv output allocation failed");
  launch_conv1d_step(ctx->in[0].as<float>(), ctx->in[1].as<float>(), ctx->in[2].as<float>(),
                     uint32_t(channels), uint32_t(kernel), ctx->out[0].as<float>(),
                     ctx->out[1].as<float>(), ctx->stream);
  if ((rc = d2h(ctx, out, ctx->out[0].p, channels * 4, "conv readback")) ||
      (rc = d2h(ctx, state_out, ctx->out[1].p, sb, "conv state readback")))
    return rc;
  return sync_and_check(ctx, "causal convolution command");
}

static int norm_impl(si_ctx* ctx, const float* x, const float* z, const float* w, uint64_t heads,
                     uint64_t hd, float eps, float* out, const char* label) {
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (heads == 0 || hd == 0 || !std::isfinite(eps) || eps <= 0.0f)
    return fail(ctx, SI_E_INVALID, std::string(label) + " dimensions are invalid");
  const uint64_t n = heads * hd;
  int rc;
  if ((rc = h2d(ctx, ctx->in[0], x, n * 4, label)) || (rc = h2d(ctx, ctx->in[1], w, hd * 4, label))) return rc;
  if (z && (rc = h2d(ctx, ctx->in[2], z, n * 4, label))) return rc;
  if (!ctx->out[0].ensure(n * 4)) return fail(ctx, SI_E_NOMEM, "norm output allocation failed");
  if (z)
    launch_rms_norm_gated(ctx->in[0].as<float>(), ctx->in[2].as<float>(), ctx->in[1].as<float>(),
                          uint32_t(heads), uint32_t(hd), eps, ctx->out[0].as<float>(), ctx->stream);
  else
    launch_rms_norm_heads(ctx->in[0].as<float>(), ctx->in[1].as<float>(), uint32_t(heads),
                          uint32_t(hd), eps, ctx->out[0].as<float>(), ctx->stream);
  if ((rc = d2h(ctx, out, ctx->out[0].p, n * 4, label))) return rc;
  return sync_and_check(ctx, label);
}

int si_rms_norm_gated(si_ctx* ctx, const float* x, const float* gate, const float* w,
                      uint64_t heads, uint64_t hd, float eps, float* out) {
  if (!ctx) return SI_E_INVALID;
  return norm_impl(ctx, x, gate, w, heads, hd, eps, out, "Gated RMSNorm");
}

int si_rms_norm_heads(si_ctx* ctx, const float* x, const float* w, uint64_t heads, uint64_t hd,
                      float eps, float* out) {
  if (!ctx) return SI_E_INVALID;
  return norm_impl(ctx, x, nullptr, w, heads, hd, eps, out, "head RMSNorm");
}

// ---- attention -------------------------------------------------------------------
}  // extern "C"

namespace si {
// Inverse RoPE frequencies theta^(-(2i)/d) computed on the host with the
// reference's expression (metal.rs:1670-1671) so device angles match it.
void rope_freqs(float theta, uint32_t dims, std::vector<float>* out) {
  out->resize(dims / 2);
  for (uint32_t i = 0; i < dims / 2; ++i) {
    const float e = (2.0f * float(i)) / float(dims);
    (*out)[i] = std::pow(theta, -e);
  }
}
}  // namespace si

extern "C" {

int si_rope(si_ctx* ctx, const float* x, uint64_t heads, uint64_t hd, uint64_t position,
            float theta, float* out) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (heads == 0 || hd == 0 || hd % 2) return fail(ctx, SI_E_INVALID, "RoPE dimensions are invalid");
  std::vector<float> f;
  rope_freqs(theta, uint32_t(hd), &f);
  const uint64_t n = heads * hd;
  int rc;
  if ((rc = h2d(ctx, ctx->in[0], x, n * 4, "rope input")) ||
      (rc = h2d(ctx, ctx->in[1], f.data(), f.size() * 4, "rope table")))
    return rc;
  if (!ctx->out[0].ensure(n * 4)) return fail(ctx, SI_E_NOMEM, "rope output allocation failed");
  launch_rope(ctx->in[0].as<float>(), ctx->in[1].as<float>(), uint32_t(heads), uint32_t(hd),
              uint32_t(position), ctx->out[0].as<float>(), ctx->stream);
  if ((rc = d2h(ctx, out, ctx->out[0].p, n * 4, "rope readback"))) return rc;
  return sync_and_check(ctx, "command");
}

int si_attention_decode(si_ctx* ctx, const si_attention_decode_input* in, float* out) {
  if (!ctx || !in) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  const uint64_t qh = in->query_heads, kvh = in->key_value_heads, hd = in->head_dim;
  if (qh > 0xffffffffull || kvh > 0xffffffffull || hd > 0xffffffffull || qh == 0 || kvh == 0 || hd == 0 ||
      qh % kvh)
    return fail(ctx, SI_E_INVALID, "attention head dimensions are invalid");
  if (hd > 256 || qh / kvh > 8)
    return fail(ctx, SI_E_UNSUPPORTED, "attention head_dim > 256 or GQA group > 8 is not supported");
  if (in->cached_tokens > in->cache_capacity_tokens || in->cache_capacity_tokens > 0xffffffffull)
    return fail(ctx, SI_E_INVALID, "attention cached token count exceeds cache capacity");
  if (in->cached_tokens + 1 > kAttnMaxTokens)
    return fail(ctx, SI_E_UNSUPPORTED, "attention over more than 1048576 tokens is not supported");
  const uint64_t esz = in->cache_type == SI_CACHE_BF16 ? 2 : 4;
  const uint64_t cache_bytes = kvh * in->cache_capacity_tokens * hd * esz;
  int rc;
  if ((rc = h2d(ctx, ctx->in[0], in->query, qh * hd * 4, "attention query")) ||
      (rc = h2d(ctx, ctx->in[1], in->key_cache, cache_bytes, "attention key cache")) ||
      (rc = h2d(ctx, ctx->in[2], in->value_cache, cache_bytes, "attention value cache")) ||
      (rc = h2d(ctx, ctx->in[3], in->new_keys, kvh * hd * 4, "attention new keys")) ||
      (rc = h2d(ctx, ctx->in[4], in->new_values, kvh * hd * 4, "attention new values")))
    return rc;
  const uint32_t chunk = 256;
  const uint64_t parts = attn_scratch_floats(uint32_t(qh), uint32_t(kvh), uint32_t(hd),
                                             uint32_t(in->cached_tokens + 1), chunk);
  if (!ctx->scratch.ensure(parts * 4) || !ctx->out[0].ensure(qh * hd * 4))
    return fail(ctx, SI_E_NOMEM, "attention scratch allocation failed");
  AttnArgs a = {};
  a.q = ctx->in[0].as<float>();
  a.k_new = ctx->in[3].as<float>();
  a.v_new = ctx->in[4].as<float>();
  a.k_cache = ctx->in[1].p;
  a.v_cache = ctx->in[2].p;
  a.cached = uint32_t(in->cached_tokens);
  a.position = 0;
  a.qh = uint32_t(qh);
  a.kvh = uint32_t(kvh);
  a.hd = uint32_t(hd);
  a.cap = uint32_t(in->cache_capacity_tokens);
  a.cache_bf16 = in->cache_type == SI_CACHE_BF16;
  a.part = ctx->scratch.as<float>();
  a.out = ctx->out[0].as<float>();
  a.chunk = chunk;
  a.err = ctx->d_err;
  launch_attention(a, ctx->stream, false);
  if ((rc = d2h(ctx, out, ctx->out[0].p, qh * hd * 4, "attention readback"))) return rc;
  return sync_and_check(ctx, "attention command");
}

int si_argmax(si_ctx* ctx, const float* logits, uint64_t n, uint32_t* index) {
  if (!ctx || !index) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (n == 0 || n > 0xffffffffull) return fail(ctx, SI_E_INVALID, "logits length is invalid");
  int rc;
  if ((rc = h2d(ctx, ctx->in[0], logits, n * 4, "argmax input"))) return rc;
  launch_argmax(ctx->in[0].as<float>(), n, ctx->d_argmax, ctx->d_index, ctx->stream);
  if ((rc = d2h(ctx, index, ctx->d_index, 4, "argmax readback"))) return rc;
  if ((rc = sync_and_check(ctx, "argmax command"))) return rc;
  if (*index == 0xffffffffu) return fail(ctx, SI_E_INVALID, "logits contain no finite values");
  return SI_OK;
}

// ---- staged layers, grouped and file-backed matvecs (metal.rs:2585-2637,
//      4780-4990, 5003-5015, 3785-3811) and allocation sampling (2374-2378) ----

static int staged_create(si_ctx* ctx, const void* packed, uint64_t bytes, uint32_t n, const char* const* names,
                         const uint64_t* starts, const uint64_t* ends, bool upload, si_staged_layer** out) {
  if (!ctx || !out) return fail(ctx, SI_E_INVALID, "invalid staged layer arguments");
  *out = nullptr;
  if (!packed || bytes == 0)
    return fail(ctx, SI_E_INVALID, upload ? "cannot promote an empty staged Qwen layer" : "cannot bind an empty staged Qwen layer");
  if (n && (!names || !starts || !ends)) return fail(ctx, SI_E_INVALID, "invalid staged layer ranges");
  auto* L = new si_staged_layer();
  L->ctx = ctx;
  L->bytes = bytes;
  uint64_t off = 0;
  for (uint32_t i = 0; i < n; ++i) {
    if (!names[i] || starts[i] > ends[i] || ends[i] > bytes) {
      delete L;
      return fail(ctx, SI_E_INVALID, std::string("staged range of ") + (names[i] ? names[i] : "?") + " is out of bounds");
    }
    L->ranges[names[i]] = {starts[i], ends[i], off};
    off = (off + (ends[i] - starts[i]) + 64 + 255) & ~uint64_t(255);  // read-ahead pad, 256-byte aligned
  }
  if (upload) {
    std::lock_guard<std::mutex> lk(ctx->upload_mu);
    cudaSetDevice(ctx->device);
    L->dev_bytes = std::max<uint64_t>(off, 256);
    cudaError_t e = fault_fire(SI_FAULT_DEVICE_ALLOC) ? cudaErrorMemoryAllocation
                                                      : cudaMalloc(reinterpret_cast<void**>(&L->dev), L->dev_bytes);
    if (e != cudaSuccess) {
      L->dev = nullptr;
      delete L;
      return cuda_fail(ctx, e, "packed Qwen layer private upload");
    }
    cudaMemsetAsync(L->dev, 0, L->dev_bytes, ctx->copy_stream);
    for (const auto& r : L->ranges)
      if (r.second.end > r.second.start)
        cudaMemcpyAsync(L->dev + r.second.dev_off, static_cast<const uint8_t*>(packed) + r.second.start,
                        r.second.end - r.second.start, cudaMemcpyHostToDevice, ctx->copy_stream);
    if ((e = cudaStreamSynchronize(ctx->copy_stream)) != cudaSuccess) {
      cudaFree(L->dev);
      delete L;
      return cuda_fail(ctx, e, "packed Qwen layer private upload");
    }
    note_alloc(ctx, int64_t(L->dev_bytes));
  } else {
    L->host = static_cast<const uint8_t*>(packed);
    if (cudaHostRegister(const_cast<void*>(packed), bytes, cudaHostRegisterReadOnly) == cudaSuccess)
      L->registered = true;
    else
      cudaGetLastError();
  }
  *out = L;
  return SI_OK;
}

int si_staged_layer_upload(si_ctx* ctx, const void* packed, uint64_t bytes, uint32_t n, const char* const* names,
                           const uint64_t* starts, const uint64_t* ends, si_staged_layer** out) {
  return staged_create(ctx, packed, bytes, n, names, starts, ends, true, out);
}

int si_staged_layer_bind_host(si_ctx* ctx, const void* packed, uint64_t bytes, uint32_t n, const char* const* names,
                              const uint64_t* starts, const uint64_t* ends, si_staged_layer** out) {
  return staged_create(ctx, packed, bytes, n, names, starts, ends, false, out);
}

int si_staged_layer_weight(const si_staged_layer* L, const char* name, uint32_t ggml_type, si_weight** out) {
  if (!L || !name || !out) return fail(L ? L->ctx : nullptr, SI_E_INVALID, "invalid staged weight arguments");
  *out = nullptr;
  auto it = L->ranges.find(name);
  if (it == L->ranges.end()) return fail(L->ctx, SI_E_INVALID, std::string("unknown staged tensor ") + name);
  auto* w = new si_weight();
  w->ctx = L->ctx;
  w->view = true;
  w->bytes = it->second.end - it->second.start;
  w->type = ggml_type;
  if (L->dev) w->dev = L->dev + it->second.dev_off;
  else w->host = L->host + it->second.start;
  *out = w;
  return SI_OK;
}

void si_staged_layer_free(si_staged_layer* L) {
  if (!L) return;
  if (L->dev) {
    cudaSetDevice(L->ctx->device);
    cudaFree(L->dev);
    note_alloc(L->ctx, -int64_t(L->dev_bytes));
  }
  if (L->registered) cudaHostUnregister(const_cast<uint8_t*>(L->host));
  delete L;
}

int si_gguf_quant_matvec_many_bytes(si_ctx* ctx, uint32_t n, const uint32_t* types, const void* const* weights,
                                    const uint64_t* nbytes, const uint64_t* rows, uint64_t cols, const float* x,
                                    float* const* ys) {
  if (!ctx) return SI_E_INVALID;
  if (n == 0) return fail(ctx, SI_E_INVALID, "staged quantized matvec group requires at least one tensor");
  if (cols == 0 || !x || !types || !weights || !nbytes || !rows || !ys)
    return fail(ctx, SI_E_INVALID, "staged quantized matvec group input length is invalid");
  for (uint32_t i = 0; i < n; ++i)
    if (int rc = si_gguf_quant_matvec_bytes(ctx, types[i], weights[i], nbytes[i], rows[i], cols, x, ys[i])) return rc;
  return SI_OK;
}

int si_f32_matvec_many(si_ctx* ctx, uint32_t n, const float* const* weights, const uint64_t* rows, uint64_t cols,
                       const float* x, float* const* ys) {
  if (!ctx) return SI_E_INVALID;
  if (n == 0) return fail(ctx, SI_E_INVALID, "GGUF F32 matvec group requires at least one tensor");
  if (cols == 0 || !x || !weights || !rows || !ys)
    return fail(ctx, SI_E_INVALID, "GGUF F32 matvec group input length is invalid");
  for (uint32_t i = 0; i < n; ++i)
    if (int rc = si_f32_matvec(ctx, weights[i], rows[i], cols, x, ys[i])) return rc;
  return SI_OK;
}

int si_gguf_matvec_tensor_rows(si_ctx* ctx, const si_gguf* g, uint64_t index, uint64_t row_start, uint64_t row_count,
                               const float* x, float* y) {
  if (!ctx || !g || !x || !y) return fail(ctx, SI_E_INVALID, "invalid tensor-rows matvec arguments");
  if (index >= g->tensors.size()) return fail(ctx, SI_E_INVALID, "GGUF tensor index out of range");
  const GgufTensor& t = g->tensors[index];
  if (t.ndim < 2) return fail(ctx, SI_E_INVALID, "tensor " + t.name + " is not a matrix");
  const uint64_t cols = t.dims[0], total_rows = t.dims[1];
  if (row_count == 0 || row_start > total_rows || row_count > total_rows - row_start)
    return fail(ctx, SI_E_INVALID, "tensor " + t.name + " rows are out of range");
  uint64_t rb;
  if (t.type == SI_GGML_TYPE_F32) {
    rb = cols * 4;
  } else if (block_bytes_of(t.type) && cols % 256 == 0) {
    rb = cols / 256 * block_bytes_of(t.type);
  } else {
    return fail(ctx, SI_E_UNSUPPORTED, "tensor " + t.name + " has no matvec for type " + std::to_string(t.type));
  }
  if (row_start + row_count > t.data_len / rb) return fail(ctx, SI_E_INVALID, "tensor " + t.name + " payload is too short");
  std::vector<uint8_t> buf(row_count * rb);
  std::string err;
  if (int rc = gguf_read(g, t.data_start + row_start * rb, buf.data(), buf.size(), &err)) return fail(ctx, rc, err);
  if (t.type == SI_GGML_TYPE_F32)
    return si_f32_matvec(ctx, reinterpret_cast<const float*>(buf.data()), row_count, cols, x, y);
  return si_gguf_quant_matvec_bytes(ctx, t.type, buf.data(), buf.size(), row_count, cols, x, y);
}

int si_gguf_quant_matvec_many_tensors(si_ctx* ctx, const si_gguf* g, uint32_t n, const uint64_t* indices,
                                      const float* x, uint64_t x_len, float* const* ys) {
  if (!ctx) return SI_E_INVALID;
  if (!g || (n && (!indices || !ys))) return fail(ctx, SI_E_INVALID, "invalid grouped tensor matvec arguments");
  if (n == 0) return fail(ctx, SI_E_INVALID, "quantized matvec group requires at least one tensor");
  for (uint32_t i = 0; i < n; ++i)
    if (indices[i] >= g->tensors.size()) return fail(ctx, SI_E_INVALID, "GGUF tensor index out of range");
  const GgufTensor& t0 = g->tensors[indices[0]];
  if (t0.ndim == 0) return fail(ctx, SI_E_INVALID, "quantized matvec tensor is not a matrix");
  const uint64_t cols = t0.dims[0];
  if (!x || x_len != cols) return fail(ctx, SI_E_INVALID, "quantized matvec group input length is invalid");
  std::vector<uint64_t> expected(n);
  for (uint32_t i = 0; i < n; ++i) {
    const GgufTensor& t = g->tensors[indices[i]];
    const uint64_t bb = block_bytes_of(t.type);
    if (t.ndim != 2 || t.dims[0] != cols || !bb)
      return fail(ctx, SI_E_INVALID, "quantized matvec group tensor shapes or types differ");
    uint64_t row_bytes = 0;
    if (__builtin_mul_overflow(cols / 256, uint64_t(bb), &row_bytes) ||
        __builtin_mul_overflow(row_bytes, t.dims[1], &expected[i]))
      return fail(ctx, SI_E_INVALID, "quantized matvec group byte length overflows");
    if (t.data_len < expected[i]) return fail(ctx, SI_E_INVALID, "quantized matvec group tensor is truncated");
  }
  std::vector<uint8_t> buf;
  std::string err;
  for (uint32_t i = 0; i < n; ++i) {
    const GgufTensor& t = g->tensors[indices[i]];
    buf.resize(expected[i]);
    if (int rc = gguf_read(g, t.data_start, buf.data(), buf.size(), &err)) return fail(ctx, rc, err);
    if (int rc = si_gguf_quant_matvec_bytes(ctx, t.type, buf.data(), buf.size(), t.dims[1], cols, x, ys[i]))
      return rc;
  }
  return SI_OK;
}

int si_gguf_dequantize_tensor(si_ctx* ctx, const si_gguf* g, uint64_t index, uint32_t type, float* out,
                              uint64_t out_len) {
  if (!ctx) return SI_E_INVALID;
  if (!g || (!out && out_len)) return fail(ctx, SI_E_INVALID, "invalid tensor dequant arguments");
  if (index >= g->tensors.size()) return fail(ctx, SI_E_INVALID, "GGUF tensor index out of range");
  const GgufTensor& t = g->tensors[index];
  const uint32_t bb = block_bytes_of(type);
  if (!bb) return fail(ctx, SI_E_UNSUPPORTED, "unsupported quantized type");
  if (t.type != type)
    return fail(ctx, SI_E_INVALID,
                type == SI_GGML_TYPE_Q4_K
                    ? "GGUF tensor " + t.name + " is not Q4_K (type " + std::to_string(t.type) + ")"
                    : "GGUF tensor " + t.name + " has type " + std::to_string(t.type) + "; expected " +
                          std::to_string(type));
  uint64_t elements = 1;
  for (uint64_t d : t.dims)
    if (__builtin_mul_overflow(elements, d, &elements))
      return fail(ctx, SI_E_INVALID, "GGUF tensor " + t.name + " element count overflows");
  if (elements % 256) return fail(ctx, SI_E_INVALID, "GGUF tensor " + t.name + " has unknown payload size");
  const uint64_t expected = elements / 256 * bb;
  if (t.data_len < expected)
    return fail(ctx, SI_E_INVALID, "GGUF tensor " + t.name + " has " + std::to_string(t.data_len) +
                                       " bytes; expected at least " + std::to_string(expected));
  if (out_len != elements) return fail(ctx, SI_E_INVALID, "dequantized output length is invalid");
  std::vector<uint8_t> buf(expected);
  std::string err;
  if (int rc = gguf_read(g, t.data_start, buf.data(), expected, &err)) return fail(ctx, rc, err);
  return si_dequantize(ctx, type, buf.data(), expected, elements, out);
}

int si_gguf_q4_k_embedding(si_ctx* ctx, const si_gguf* g, uint64_t index, uint64_t token, float* out) {
  if (!ctx || !g || !out) return fail(ctx, SI_E_INVALID, "invalid embedding arguments");
  if (index >= g->tensors.size()) return fail(ctx, SI_E_INVALID, "GGUF tensor index out of range");
  const GgufTensor& t = g->tensors[index];
  if (t.type != SI_GGML_TYPE_Q4_K || t.ndim != 2) return fail(ctx, SI_E_INVALID, "Q4_K embedding requires a rank-2 Q4_K tensor");
  const uint64_t cols = t.dims[0], rows = t.dims[1];
  if (token >= rows || cols % 256) return fail(ctx, SI_E_INVALID, "Q4_K embedding token id or dimension is invalid");
  const uint64_t rb = cols / 256 * 144;
  if ((token + 1) * rb > t.data_len) return fail(ctx, SI_E_INVALID, "Q4_K embedding row exceeds the tensor payload");
  std::vector<uint8_t> row(rb);
  std::string err;
  if (int rc = gguf_read(g, t.data_start + token * rb, row.data(), rb, &err)) return fail(ctx, rc, err);
  return si_q4_k_embedding_row(ctx, row.data(), rb, cols, out);
}

int si_fault_inject(uint32_t site, uint32_t skip) {
  if (site >= si::SI_FAULT_SITES) return si::fail(nullptr, SI_E_INVALID, "unknown fault site " + std::to_string(site));
  if (site == 0) {
    for (auto& f : si::g_fault) f.store(-1);
    return SI_OK;
  }
  si::g_fault[site].store(int64_t(skip));
  return SI_OK;
}

int si_sample_allocated(si_ctx* ctx) {
  if (!ctx) return SI_E_INVALID;
  const uint64_t cur = ctx->allocated.load();
  uint64_t peak = ctx->peak_allocated.load();
  while (cur > peak && !ctx->peak_allocated.compare_exchange_weak(peak, cur)) {
  }
  return SI_OK;
}

}  // extern "C"
