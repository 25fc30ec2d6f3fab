// Peer buffers and the row-sharded matvec whose all-gather runs inside the
// matvec kernel.
//
// A peer buffer is one device allocation per rank of a context's communicator,
// mapped into every other rank with CUDA IPC (the handles travel over NCCL),
// laid out as
//   [0, D)                   data (D = the requested bytes rounded up to 256)
//   [D + 512, D + 516)       this rank's CTA ticket of the in-kernel exchange
//   [D + 576, D + 580)       launches of the in-kernel exchange so far (epoch)
//   [D + 1536, D + 2048)     flags of the stand-alone peer all-gather (fallback)
//   [D + 2560, D + 2560 + 4D) exchange words: two parity halves of D/4 8-byte
//                            words, word i standing for float i of the data
// si_sharded_qmatvec_dev runs the Q4_K (or, for the shapes it takes, the Q6_K)
// tensor-core matvec on this rank's rows;
// its epilogue stores each row, tagged with the launch's epoch, into every
// rank's exchange words over NVLink, and each CTA unpacks its slice of the
// gathered vector into the data once every rank's rows have arrived, so the
// launch completes with the whole vector on every rank (PeerOut in
// qmatvec.cuh). Other types, and shapes that kernel does
// not take, run the matvec into the local slice and then the stand-alone
// peer all-gather kernel (one launch more).
//
// Row sharding of a matvec is the BASELINE's multi-GPU partitioning of the
// reference's single-GPU matvec (src/metal.rs:3357-3397, 3923); the reference
// itself has no multi-GPU path.
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "../../include/si_cuda.h"
#include "comm.h"
#include "common.cuh"
#include "ctx.h"
#include "kernels.cuh"
#include "qmatvec.cuh"

struct si_peer_buffer {
  si_ctx* ctx = nullptr;
  int n = 1, rank = 0;
  uint64_t bytes = 0, data_bytes = 0;
  void* peers[si::kPeerMax] = {};
  std::vector<void*> owned;   // allocations made here (one, or every emulated rank's)
  bool ipc = false;           // peers[] other than this rank's are IPC mappings
  uint32_t host_epoch = 0;    // epochs of the stand-alone all-gather
  long long wait_cycles = si::kWaitCycles;
};

namespace {

constexpr uint64_t kTicketOff = 512, kEpochOff = 576, kFlagOff = 1536, kTail = 2560;

// bytes of one rank's allocation: data, tail, exchange words
uint64_t alloc_bytes(uint64_t data_bytes) { return data_bytes + kTail + 4 * data_bytes; }

uint64_t round256(uint64_t v) { return (v + 255) & ~255ull; }

int alloc_zeroed(si_ctx* ctx, uint64_t bytes, void** out) {
  cudaError_t e = cudaMalloc(out, bytes);
  if (e != cudaSuccess) return si::fail(ctx, SI_E_NOMEM, std::string("peer buffer allocation: ") + cudaGetErrorString(e));
  if ((e = cudaMemset(*out, 0, bytes)) != cudaSuccess) {
    cudaFree(*out);
    return si::cuda_fail(ctx, e, "peer buffer clear");
  }
  si::note_alloc(ctx, int64_t(bytes));
  return SI_OK;
}

}  // namespace

extern "C" {

int si_peer_buffer_create(si_ctx* ctx, uint64_t bytes, si_peer_buffer** out) {
  if (!ctx || !out || bytes == 0) return si::fail(ctx, SI_E_INVALID, "invalid peer buffer arguments");
  *out = nullptr;
  if (ctx->nranks > si::kPeerMax) return si::fail(ctx, SI_E_UNSUPPORTED, "peer buffers span at most 8 ranks");
  std::lock_guard<std::mutex> lk(ctx->mu);
  cudaSetDevice(ctx->device);
  auto* b = new si_peer_buffer();
  b->ctx = ctx;
  b->n = ctx->nranks;
  b->rank = ctx->rank;
  b->bytes = bytes;
  b->data_bytes = round256(bytes);
  void* local = nullptr;
  if (int rc = alloc_zeroed(ctx, alloc_bytes(b->data_bytes), &local)) {
    delete b;
    return rc;
  }
  b->owned.push_back(local);
  if (b->n > 1) {
    // every rank's allocation is cleared before any rank can store into it
    cudaDeviceSynchronize();
    if (int rc = si::comm_p2p_map(ctx, local, b->peers)) {
      si_peer_buffer_destroy(b);
      return rc;
    }
    b->ipc = true;
  } else {
    b->peers[0] = local;
  }
  *out = b;
  return SI_OK;
}

int si_peer_buffer_create_local(si_ctx* ctx, uint64_t bytes, uint32_t nranks, uint32_t rank, uint64_t wait_us,
                                si_peer_buffer** out) {
  if (!ctx || !out || bytes == 0 || nranks == 0 || nranks > uint32_t(si::kPeerMax) || rank >= nranks)
    return si::fail(ctx, SI_E_INVALID, "invalid peer buffer arguments");
  *out = nullptr;
  std::lock_guard<std::mutex> lk(ctx->mu);
  cudaSetDevice(ctx->device);
  auto* b = new si_peer_buffer();
  b->ctx = ctx;
  b->n = int(nranks);
  b->rank = int(rank);
  b->bytes = bytes;
  b->data_bytes = round256(bytes);
  // about 2,000 SM cycles per microsecond (the clock is at most 1,965 MHz)
  if (wait_us) b->wait_cycles = (long long)(wait_us < 1000000000ull ? wait_us : 1000000000ull) * 2000;
  for (uint32_t p = 0; p < nranks; ++p) {
    void* m = nullptr;
    if (int rc = alloc_zeroed(ctx, alloc_bytes(b->data_bytes), &m)) {
      si_peer_buffer_destroy(b);
      return rc;
    }
    b->owned.push_back(m);
    b->peers[p] = m;
  }
  cudaDeviceSynchronize();
  *out = b;
  return SI_OK;
}

void si_peer_buffer_destroy(si_peer_buffer* b) {
  if (!b) return;
  cudaSetDevice(b->ctx->device);
  cudaDeviceSynchronize();
  if (b->ipc) si::comm_p2p_unmap(b->ctx, b->peers);
  for (void* m : b->owned) {
    cudaFree(m);
    si::note_alloc(b->ctx, -int64_t(alloc_bytes(b->data_bytes)));
  }
  delete b;
}

void* si_peer_buffer_local(const si_peer_buffer* b) { return b ? b->peers[b->rank] : nullptr; }

int si_sharded_qmatvec_dev(si_ctx* ctx, si_peer_buffer* b, uint32_t type, const void* w_shard,
                           uint64_t rows_per_rank, uint64_t cols, const float* x, uint64_t y_offset, void* stream) {
  if (!ctx || !b || b->ctx != ctx || !w_shard || !x) return si::fail(ctx, SI_E_INVALID, "invalid sharded matvec arguments");
  const uint32_t bb = si::block_bytes_of(type);
  if (bb == 0) return si::fail(ctx, SI_E_UNSUPPORTED, "unsupported quantized weight type");
  if (rows_per_rank == 0 || cols == 0 || cols % 256 || cols > si::kQmvMaxCols || rows_per_rank > 0xffffffffull)
    return si::fail(ctx, SI_E_INVALID, "sharded matvec dimensions are invalid");
  if (y_offset % 16 || y_offset + uint64_t(b->n) * rows_per_rank * 4 > b->data_bytes)
    return si::fail(ctx, SI_E_INVALID, "the gathered vector does not fit the peer buffer (or is not 16-byte aligned)");
  const cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const uint64_t slice = y_offset + uint64_t(b->rank) * rows_per_rank * 4;
  si::QmvParams p = {};
  p.type = type;
  p.cols = uint32_t(cols);
  p.nseg = 1;
  p.seg[0] = {static_cast<const uint8_t*>(w_shard), reinterpret_cast<float*>(static_cast<uint8_t*>(b->peers[b->rank]) + slice),
              nullptr, uint32_t(rows_per_rank), 0};
  p.items = uint32_t(rows_per_rank);
  p.xmode = si::XM_RAW;
  p.x = x;
  p.err = ctx->d_err;
  si::qscratch_for(ctx, s, &p.scratch, &p.scratch_bytes);
  std::string msg;
  int rc;
  if (b->n == 1) {
    rc = si::launch_qmv(p, s, ctx->sm_count, true, &msg);
  } else {
    si::QmvParams q = p;
    q.peer.n = uint32_t(b->n);
    q.peer.rank = uint32_t(b->rank);
    for (int r = 0; r < b->n; ++r) {
      uint8_t* base = static_cast<uint8_t*>(b->peers[r]);
      q.peer.ll[r] = reinterpret_cast<uint64_t*>(base + b->data_bytes + kTail) + y_offset / 4;
    }
    uint8_t* mine = static_cast<uint8_t*>(b->peers[b->rank]);
    q.peer.parity_stride = b->data_bytes / 4;
    q.peer.y = reinterpret_cast<float*>(mine + y_offset);
    q.peer.row0 = uint32_t(uint64_t(b->rank) * rows_per_rank);
    q.peer.total = uint32_t(uint64_t(b->n) * rows_per_rank);
    q.peer.ticket = reinterpret_cast<uint32_t*>(mine + b->data_bytes + kTicketOff);
    q.peer.epoch = reinterpret_cast<uint32_t*>(mine + b->data_bytes + kEpochOff);
    q.peer.wait_cycles = b->wait_cycles;
    if (type == SI_GGML_TYPE_Q6_K)
      rc = si::qmv_tc6_eligible(q) ? si::launch_qmv_tc6(q, s, ctx->sm_count, true, &msg) : SI_E_UNSUPPORTED;
    else
      rc = si::qmv_tc_supported(q) ? si::launch_qmv_tc(q, s, ctx->sm_count, true, &msg) : SI_E_UNSUPPORTED;
    if (rc == SI_E_UNSUPPORTED) {
      // the matvec into this rank's slice, then the stand-alone peer all-gather
      rc = si::launch_qmv(p, s, ctx->sm_count, true, &msg);
      if (!rc) {
        si::P2PGather g = {};
        for (int r = 0; r < b->n; ++r) g.block[r] = static_cast<uint8_t*>(b->peers[r]);
        g.send[0] = p.seg[0].y;
        g.recv_off[0] = y_offset;
        g.count[0] = uint32_t(rows_per_rank);
        g.n = uint32_t(b->n);
        g.rank = uint32_t(b->rank);
        g.epoch = ++b->host_epoch;
        g.flag_off = b->data_bytes + kFlagOff;
        g.err = ctx->d_err;
        g.wait_cycles = b->wait_cycles;
        si::launch_p2p_allgather(g, s);
      }
    }
  }
  if (rc) return si::fail(ctx, rc, msg);
  if (cudaError_t e = cudaGetLastError()) return si::cuda_fail(ctx, e, "sharded matvec launch");
  si::note_async_submission(ctx);
  return SI_OK;
}

int si_ctx_synchronize(si_ctx* ctx) {
  if (!ctx) return SI_E_INVALID;
  std::lock_guard<std::mutex> lk(ctx->mu);
  cudaSetDevice(ctx->device);
  return si::sync_and_check(ctx, "synchronize");
}

}  // extern "C"
