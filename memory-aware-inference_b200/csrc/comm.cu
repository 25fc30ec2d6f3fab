// NCCL communicator attached to a context: one process per GPU, row-sharded
// weights. NCCL carries set-up (including the exchange of CUDA IPC handles
// that maps every rank's model scratch into its peers, for the NVLink
// peer-store all-gathers of kernels.cu) and the collectives that stay on it.
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "comm.h"
#include "ctx.h"

using namespace si;

struct si_comm_state {
  ncclComm_t comm = nullptr;
};

namespace si {

// Poll a non-blocking NCCL operation until it leaves ncclInProgress, bounded
// by `seconds`; on timeout the communicator is aborted. Collective enqueues
// settle within microseconds, so the first millisecond spins (yielding the
// core) and only longer waits (communicator set-up) sleep between polls.
static ncclResult_t wait_nccl(ncclComm_t comm, double seconds) {
  auto t0 = std::chrono::steady_clock::now();
  ncclResult_t st = ncclInProgress;
  while (true) {
    ncclResult_t r = ncclCommGetAsyncError(comm, &st);
    if (r != ncclSuccess) return r;
    if (st != ncclInProgress) return st;
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > seconds) return ncclInProgress;
    if (el < 1e-3)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// A non-blocking communicator may return ncclInProgress from an enqueue; the
// next call must not start before it reports success. Bounded wait (the
// enqueue itself, not the GPU work); on timeout the communicator is aborted.
static int settle(si_ctx* ctx, ncclResult_t r, const char* what) {
  if (r == ncclInProgress) r = wait_nccl(ctx->comm->comm, 60.0);
  if (r == ncclInProgress) {
    ncclCommAbort(ctx->comm->comm);
    delete ctx->comm;
    ctx->comm = nullptr;
    return fail(ctx, SI_E_TIMEOUT, std::string(what) + ": communicator did not become ready; aborted");
  }
  if (r != ncclSuccess) return fail(ctx, SI_E_COMM, std::string(what) + ": " + ncclGetErrorString(r));
  return SI_OK;
}

int comm_allgather(si_ctx* ctx, const float* send, float* recv, size_t count, cudaStream_t s) {
  if (!ctx->comm) return SI_OK;
  return settle(ctx, ncclAllGather(send, recv, count, ncclFloat32, ctx->comm->comm, s), "ncclAllGather");
}

// Two all-gathers issued as one NCCL group: one launch, one latency.
int comm_allgather2(si_ctx* ctx, const float* s1, float* r1, size_t n1, const float* s2, float* r2, size_t n2,
                    cudaStream_t s) {
  if (!ctx->comm) return SI_OK;
  ncclComm_t c = ctx->comm->comm;
  ncclResult_t r = ncclGroupStart();
  if (r == ncclSuccess) r = ncclAllGather(s1, r1, n1, ncclFloat32, c, s);
  if (r == ncclSuccess || r == ncclInProgress) r = ncclAllGather(s2, r2, n2, ncclFloat32, c, s);
  const ncclResult_t e = ncclGroupEnd();
  if (r == ncclSuccess || r == ncclInProgress) r = e;
  return settle(ctx, r, "ncclAllGather (grouped)");
}

// Map a device allocation of every rank into this process: the CUDA IPC
// handles of `base` travel over the communicator; peers[rank] = base.
int comm_p2p_map(si_ctx* ctx, void* base, void** peers) {
  const int n = ctx->nranks, r = ctx->rank;
  if (!ctx->comm || n < 2) return SI_E_STATE;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) return fail(ctx, SI_E_CUDA, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  constexpr size_t HB = sizeof(cudaIpcMemHandle_t);
  uint8_t* dh = nullptr;
  if ((e = cudaMalloc(&dh, HB * n)) != cudaSuccess)
    return fail(ctx, SI_E_NOMEM, std::string("IPC handle exchange buffer: ") + cudaGetErrorString(e));
  std::vector<uint8_t> all(HB * n);
  cudaMemcpyAsync(dh + HB * r, &h, HB, cudaMemcpyHostToDevice, ctx->stream);
  int rc = settle(ctx, ncclAllGather(dh + HB * r, dh, HB, ncclUint8, ctx->comm->comm, ctx->stream),
                  "ncclAllGather(IPC handles)");
  if (!rc) {
    cudaMemcpyAsync(all.data(), dh, HB * n, cudaMemcpyDeviceToHost, ctx->stream);
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) rc = fail(ctx, SI_E_CUDA, std::string("IPC handle exchange: ") + cudaGetErrorString(e));
  }
  cudaFree(dh);
  if (rc) return rc;
  for (int p = 0; p < n; ++p) {
    if (p == r) {
      peers[p] = base;
      continue;
    }
    cudaIpcMemHandle_t hp;
    std::memcpy(&hp, all.data() + HB * p, HB);
    e = cudaIpcOpenMemHandle(&peers[p], hp, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < p; ++q)
        if (q != r) cudaIpcCloseMemHandle(peers[q]);
      return fail(ctx, SI_E_CUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
    }
  }
  return SI_OK;
}

void comm_p2p_unmap(si_ctx* ctx, void** peers) {
  for (int p = 0; p < ctx->nranks; ++p)
    if (p != ctx->rank && peers[p]) cudaIpcCloseMemHandle(peers[p]);
}

int comm_allreduce_sum(si_ctx* ctx, const float* send, float* recv, size_t count, cudaStream_t s) {
  if (!ctx->comm) return SI_OK;
  return settle(ctx, ncclAllReduce(send, recv, count, ncclFloat32, ncclSum, ctx->comm->comm, s), "ncclAllReduce");
}

int comm_allgather_u64(si_ctx* ctx, const unsigned long long* send, unsigned long long* recv,
                       cudaStream_t s) {
  if (!ctx->comm) return SI_OK;
  return settle(ctx, ncclAllGather(send, recv, 1, ncclUint64, ctx->comm->comm, s), "ncclAllGather(u64)");
}

void comm_destroy(si_ctx* ctx) {
  if (!ctx || !ctx->comm) return;
  ncclCommDestroy(ctx->comm->comm);
  delete ctx->comm;
  ctx->comm = nullptr;
}

}  // namespace si

extern "C" {

int si_comm_unique_id(void* id_out) {
  if (!id_out) return SI_E_INVALID;
  static_assert(sizeof(ncclUniqueId) <= SI_COMM_ID_BYTES, "NCCL id size");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return fail(nullptr, SI_E_COMM, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
  std::memset(id_out, 0, SI_COMM_ID_BYTES);
  std::memcpy(id_out, &id, sizeof(id));
  return SI_OK;
}

int si_ctx_comm_init(si_ctx* ctx, int nranks, int rank, const void* id) {
  if (!ctx || !id || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(ctx, SI_E_INVALID, "invalid communicator arguments");
  if (ctx->comm) return fail(ctx, SI_E_STATE, "communicator already initialised");
  if (nranks == 1) {
    ctx->nranks = 1;
    ctx->rank = 0;
    return SI_OK;
  }
  cudaSetDevice(ctx->device);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  auto* st = new si_comm_state();
  ncclResult_t r = ncclCommInitRankConfig(&st->comm, nranks, uid, rank, &cfg);
  if (r == ncclInProgress) r = wait_nccl(st->comm, 120.0);
  if (r != ncclSuccess) {
    if (st->comm) ncclCommAbort(st->comm);
    delete st;
    return fail(ctx, SI_E_COMM, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
  }
  ctx->comm = st;
  ctx->nranks = nranks;
  ctx->rank = rank;
  return SI_OK;
}

int si_ctx_comm_info(const si_ctx* ctx, int* nranks, int* rank) {
  if (!ctx) return SI_E_INVALID;
  if (nranks) *nranks = ctx->nranks;
  if (rank) *rank = ctx->rank;
  return SI_OK;
}

}  // extern "C"
