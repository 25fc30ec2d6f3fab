// Device side of the in-kernel all-gather of a row-sharded matvec (PeerOut,
// qmatvec.cuh), shared by the Q4_K and Q6_K tensor-core kernels: each output
// row leaves as one 8-byte {value, epoch} word for every rank, and every CTA
// then unpacks its slice of the gathered vector as the words arrive.
#pragma once
#include <cstdint>

#include "common.cuh"
#include "qmatvec.cuh"

namespace si {

// The slice of CTA `cta` (of `nctas`) of the gathered vector, word by word,
// as soon as each word carries this launch's epoch (bounded), unpacked into
// y; thread `tid` of `nthreads` takes every nthreads-th word. No barrier.
static __device__ __forceinline__ void peer_unpack(const PeerOut& po, uint32_t cta, uint32_t nctas, uint32_t epoch,
                                                   int* err, uint32_t tid, uint32_t nthreads) {
  const uint32_t lo = uint32_t(uint64_t(cta) * po.total / nctas);
  const uint32_t hi = uint32_t(uint64_t(cta + 1) * po.total / nctas);
  const uint64_t* w = po.ll[po.rank] + (epoch & 1) * po.parity_stride;
  const long long t0 = clock64();
  for (uint32_t i = lo + tid; i < hi; i += nthreads) {
    uint64_t v;
    while (true) {
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w + i) : "memory");
      if (uint32_t(v >> 32) == epoch) break;
      if (clock64() - t0 > po.wait_cycles) break;
    }
    if (uint32_t(v >> 32) != epoch) {
      if (err) atomicOr(err, KERR_TIMEOUT_FULL);
      break;
    }
    po.y[i] = __uint_as_float(uint32_t(v));
  }
}

// After the CTA's unpacking (all `nthreads` threads, named barrier 1): the
// CTA's ticket, the launch's last CTA resetting it and advancing the epoch.
static __device__ __forceinline__ void peer_ticket(const PeerOut& po, uint32_t nctas, uint32_t epoch, uint32_t tid,
                                                   uint32_t nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
  if (tid == 0) {
    // every CTA has read the epoch (at its start) before the last ticket
    if (atomicAdd(po.ticket, 1u) == nctas - 1) {
      *po.ticket = 0;
      asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(po.epoch), "r"(epoch) : "memory");
    }
  }
}

// After the CTA's own rows have gone out, called by all `nthreads` consumer
// threads of a 1-D grid: its slice of the gathered vector, then its ticket.
static __device__ __noinline__ void peer_gather(const PeerOut& po, uint32_t nctas, uint32_t epoch, int* err,
                                                uint32_t nthreads) {
  peer_unpack(po, blockIdx.x, nctas, epoch, err, threadIdx.x, nthreads);
  peer_ticket(po, nctas, epoch, threadIdx.x, nthreads);
}

static __device__ __forceinline__ void peer_store_row(const PeerOut& po, uint32_t epoch, uint32_t row, float v) {
  const uint64_t word = (uint64_t(epoch) << 32) | __float_as_uint(v);
  const uint64_t at = (epoch & 1) * po.parity_stride + po.row0 + row;
  for (uint32_t p = 0; p < po.n; ++p)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(po.ll[p] + at), "l"(word) : "memory");
}

}  // namespace si
