// Collectives used by the row-sharded model (no-ops without a communicator).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

struct si_ctx;

namespace si {
int comm_allgather(si_ctx* ctx, const float* send, float* recv, size_t count, cudaStream_t s);
int comm_allgather2(si_ctx* ctx, const float* s1, float* r1, size_t n1, const float* s2, float* r2, size_t n2,
                    cudaStream_t s);
int comm_allreduce_sum(si_ctx* ctx, const float* send, float* recv, size_t count, cudaStream_t s);
int comm_allgather_u64(si_ctx* ctx, const unsigned long long* send, unsigned long long* recv,
                       cudaStream_t s);
// CUDA IPC mapping of one device allocation of every rank (peers[nranks];
// peers[rank] is `base` itself), exchanged over the communicator.
int comm_p2p_map(si_ctx* ctx, void* base, void** peers);
void comm_p2p_unmap(si_ctx* ctx, void** peers);
// Destroy the context's communicator, if any (context teardown).
void comm_destroy(si_ctx* ctx);
}  // namespace si
