// Split-K attention decode that allocates nothing.
//
// Who needs it: callers that must not (or cannot) allocate device memory at
// call time -- code running while a stream is being captured into a CUDA
// graph, code inside a memory-pool-less embedding runtime that forbids
// cudaMalloc after start-up, or a host whose allocator is shared and locked by
// someone else. They pass device inputs and an output buffer; the split-K
// partial results live in a fixed array inside this library instead of in a
// buffer allocated per call.
//
// Limits and sharing: the array holds kNoAllocPartFloats floats (4 MiB) on
// every GPU that loads the library, for the life of the process. A call whose
// partials would not fit is rejected. All calls on a device share the array,
// so calls that overlap on the GPU (different streams, no ordering between
// them) race on it. Every partial that the combine step reads is written by
// the same call first, so nothing has to be cleared between calls.
//
// Set-up: the first call on a device, with that device current, looks up the
// array's device address (cudaGetSymbolAddress); make that first call before
// any stream capture on the device. Calls made outside a capture look the
// address up again, so a device reset or a new primary context never leaves a
// stale address behind; calls made during a capture use the last one found.
//
// Timed-out waits: the tensor-core split kernel bounds its waits for staged
// K/V tiles (about 2 s of SM clocks). A split whose wait runs out contributes
// nothing and sets a bit in a device error word kept beside the scratch. A
// later call made outside a capture whose stream has drained reads and clears
// that word and returns SI_E_TIMEOUT for the earlier call's failure (its own
// work is not enqueued); while the stream is still busy the check is skipped,
// so the report can come one or more calls late.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/si_cuda.h"
#include "kernels.cuh"

namespace si {
int fail(si_ctx* ctx, int code, const std::string& msg);
}

namespace {

constexpr size_t kNoAllocPartFloats = size_t(1) << 20;  // 4 MiB of partials
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_attn_parts[kNoAllocPartFloats];
static __device__ int g_attn_err;  // timed-out waits of earlier calls (bits)

std::mutex g_mu;
float* g_parts_ptr[kMaxDevices] = {};
int* g_err_ptr[kMaxDevices] = {};

// Device addresses of g_attn_parts and g_attn_err on the current device. The
// lookup is repeated outside a capture (cheap, and it follows a device reset);
// inside a capture the addresses from the last lookup are used.
int scratch_ptrs(cudaStream_t stream, bool capturing, float** parts, int** err) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return si::fail(nullptr, SI_E_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return si::fail(nullptr, SI_E_UNSUPPORTED, "device ordinal out of range");
  (void)stream;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!capturing || !g_parts_ptr[dev]) {
    if (capturing)
      return si::fail(nullptr, SI_E_UNSUPPORTED,
                      "the first allocation-free attention call on a device must come before any stream capture");
    void* p = nullptr;
    void* q = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_parts);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&q, g_attn_err);
    if (e != cudaSuccess || !p || !q)
      return si::fail(nullptr, SI_E_CUDA,
                      std::string("cudaGetSymbolAddress(attention scratch): ") + cudaGetErrorString(e));
    g_parts_ptr[dev] = static_cast<float*>(p);
    g_err_ptr[dev] = static_cast<int*>(q);
  }
  *parts = g_parts_ptr[dev];
  *err = g_err_ptr[dev];
  return SI_OK;
}

}  // namespace

extern "C" int si_attention_decode_noalloc_dev(const si_attention_decode_input* in, float* out,
                                               void* stream) {
  if (!in || !out || !in->query || !in->key_cache || !in->value_cache || !in->new_keys ||
      !in->new_values)
    return si::fail(nullptr, SI_E_INVALID, "attention arguments are null");
  const uint64_t qh = in->query_heads, kvh = in->key_value_heads, hd = in->head_dim;
  if (qh > 0xffffffffull || kvh > 0xffffffffull || hd > 0xffffffffull)
    return si::fail(nullptr, SI_E_INVALID, "attention head dimensions are invalid");
  if (qh == 0 || kvh == 0 || hd == 0 || qh % kvh)
    return si::fail(nullptr, SI_E_INVALID, "attention head dimensions are invalid");
  if (hd > 256 || qh / kvh > 8)
    return si::fail(nullptr, SI_E_UNSUPPORTED, "attention head_dim > 256 or GQA group > 8 is not supported");
  if (in->cached_tokens > in->cache_capacity_tokens || in->cache_capacity_tokens > 0xffffffffull)
    return si::fail(nullptr, SI_E_INVALID, "attention cached token count exceeds cache capacity");
  if (in->cached_tokens + 1 > si::kAttnMaxTokens)
    return si::fail(nullptr, SI_E_UNSUPPORTED, "attention over more than 1048576 tokens is not supported");
  const uint32_t chunk = 256;
  const uint64_t need = si::attn_scratch_floats(uint32_t(qh), uint32_t(kvh), uint32_t(hd), uint32_t(in->cached_tokens + 1), chunk);
  if (need > kNoAllocPartFloats)
    return si::fail(nullptr, SI_E_UNSUPPORTED,
                    "attention needs " + std::to_string(need) + " scratch floats; the allocation-free entry point holds " +
                        std::to_string(kNoAllocPartFloats) + " (fewer cached tokens or heads required)");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaError_t e = cudaStreamIsCapturing(st, &cap))
    return si::fail(nullptr, SI_E_CUDA, std::string("cudaStreamIsCapturing: ") + cudaGetErrorString(e));
  const bool capturing = cap != cudaStreamCaptureStatusNone;
  float* parts = nullptr;
  int* err = nullptr;
  if (int rc = scratch_ptrs(st, capturing, &parts, &err)) return rc;
  // report a timed-out wait of an earlier call, when that costs no waiting
  if (!capturing && cudaStreamQuery(st) == cudaSuccess) {
    int h = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_attn_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && h) {
      const int zero = 0;
      e = cudaMemcpyToSymbolAsync(g_attn_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(st);
      if (e == cudaSuccess)
        return si::fail(nullptr, SI_E_TIMEOUT,
                        "an earlier allocation-free attention call timed out waiting for K/V tiles (error bits " +
                            std::to_string(h) + "); its output is incomplete");
    }
    if (e != cudaSuccess)
      return si::fail(nullptr, SI_E_CUDA, std::string("attention error word: ") + cudaGetErrorString(e));
  }
  si::AttnArgs a = {};
  a.q = in->query;
  a.k_new = in->new_keys;
  a.v_new = in->new_values;
  a.k_cache = in->key_cache;
  a.v_cache = in->value_cache;
  a.cached = uint32_t(in->cached_tokens);
  a.qh = uint32_t(qh);
  a.kvh = uint32_t(kvh);
  a.hd = uint32_t(hd);
  a.cap = uint32_t(in->cache_capacity_tokens);
  a.cache_bf16 = in->cache_type == SI_CACHE_BF16;
  a.part = parts;
  a.out = out;
  a.chunk = chunk;
  a.err = err;
  si::launch_attention(a, st, false);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return si::fail(nullptr, SI_E_CUDA, std::string("attention launch: ") + cudaGetErrorString(e));
  return SI_OK;
}
