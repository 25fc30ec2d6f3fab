// Internal definition of the backend context shared by the C-ABI files.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <vector>
#include <string>

#include "../../include/si_cuda.h"

struct si_comm_state;

namespace si {

// Grow-only device buffer used as per-call staging for host-memory calls.
struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
  }
  // Ensures `bytes` (+64 B read-ahead padding for the bulk copies).
  bool ensure(size_t bytes) {
    if (bytes + 64 <= cap) return true;
    release();
    size_t want = bytes + 64;
    if (cudaMalloc(&p, want) != cudaSuccess) {
      p = nullptr;
      return false;
    }
    cap = want;
    return true;
  }
  template <typename T>
  T* as() const { return static_cast<T*>(p); }
};

// Whole-layer retention policy of the models created on a context
// (si_ctx_set_retention); `set` false = the budget-filled prefix.
struct Retention {
  bool set = false;
  uint32_t prefix = 0, stride = 0, offset = 0, flags = 0;
  std::vector<uint32_t> layers;
  // tensor-level forms (SI_RETAIN_TENSORS; si_retention in si_cuda.h)
  uint32_t mlp_layers = 0, mlp_stride = 0, mlp_offset = 0, q6_layers = 0;
  uint32_t down_stride = 0, down_offset = 0, attention_stride = 0, attention_offset = 0;
};

}  // namespace si

struct si_ctx {
  int device = 0;
  int sm_count = 0;
  si_ctx_config cfg{};
  cudaStream_t stream = nullptr;       // compute
  cudaStream_t copy_stream = nullptr;  // weight staging
  int* d_err = nullptr;                // kernel error bits
  int* h_err = nullptr;                // pinned copy of d_err, read after each sync
  // Pinned staging for the readbacks of one host-memory call: the copies are
  // enqueued into it and copied to the caller's memory after the sync.
  struct PendingCopy {
    void* dst;
    size_t off, bytes;
  };
  uint8_t* h_stage = nullptr;
  size_t h_stage_cap = 0, h_stage_used = 0;
  std::vector<PendingCopy> pending;
  unsigned long long* d_argmax = nullptr;
  uint32_t* d_index = nullptr;
  std::string err;
  std::mutex mu;         // serialises host-memory entry points
  std::mutex upload_mu;  // serialises weight uploads from staging threads
  si::DevBuf in[6], out[3], wbuf[3], scratch;
  // partial sums of the matvec rows whose blocks span several CTAs, and the
  // per-group counters (zero between launches): kQmvScratchSlots slots, slot 0
  // for the context's stream, the others handed to the first other streams
  // that launch a matvec (a slot is never shared by two streams, so launches
  // on different streams cannot meet in it)
  si::DevBuf qscratch;
  std::mutex qs_mu;
  cudaStream_t qs_stream[8] = {};
  // telemetry
  std::atomic<uint64_t> allocated{0}, peak_allocated{0}, peak_weights{0}, weights{0};
  std::atomic<uint64_t> peak_kv{0}, peak_scratch{0}, submitted{0}, waited{0}, wait_nanos{0}, async_submitted{0};
  // NCCL (optional)
  si_comm_state* comm = nullptr;
  int nranks = 1, rank = 0;
  si::Retention retention;
};

namespace si {
int fail(si_ctx* ctx, int code, const std::string& msg);
int cuda_fail(si_ctx* ctx, cudaError_t e, const char* what);
// Synchronise the compute stream and convert kernel error bits to a status.
int sync_and_check(si_ctx* ctx, const char* what);
void note_alloc(si_ctx* ctx, int64_t delta);
void note_weights(si_ctx* ctx, int64_t delta);
void note_async_submission(si_ctx* ctx);
// The split-group scratch slot of `stream` (null: none is free; the matvec
// then runs without it).
void qscratch_for(si_ctx* ctx, cudaStream_t stream, void** p, uint64_t* bytes);
}  // namespace si
