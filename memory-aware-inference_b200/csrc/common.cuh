// Shared device helpers for the sm_100a decode kernels: mbarrier-tracked
// bulk async copies (the non-tensor TMA path), bounded waits, programmatic
// dependent launch, warp reductions and GGUF field decoding.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/si_cuda.h"

namespace si {

// Error bits written by kernels into the context's device error word.
enum : int {
  KERR_TIMEOUT_FULL = 1,   // a consumer gave up waiting for a staged tile
  KERR_TIMEOUT_EMPTY = 2,  // the producer gave up waiting for a free slot
  KERR_TIMEOUT_DRAIN = 4,  // copies still in flight at exit after a timeout
  KERR_BAD_INDEX = 8,      // an index checked on the device was out of range
};

// Every device-side wait is bounded by this many SM clock cycles (~2 s at
// 1.9 GHz). A wait that runs out records an error bit and returns false.
constexpr long long kWaitCycles = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with `parity` to complete.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitCycles) return false;
  }
  return true;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Non-tensor bulk copy global -> shared, completion signalled on `bar` as
// transaction bytes. dst/src 16-byte aligned, bytes a multiple of 16. No
// multicast: the source is always this GPU's own memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 prefetch of `bytes` (multiple of 16) at a 16-byte aligned address.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue (weight prefetch) while this one drains; block until the previous
// kernel's results are visible before touching activations.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float as_f(uint32_t u) { return __uint_as_float(u); }

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

// Scale/min pair `index` of the 12-byte packed 6-bit table (GGUF K-quants).
__device__ __forceinline__ void scale_min_k4(int index, const uint8_t* s, uint32_t& sc,
                                             uint32_t& mn) {
  if (index < 4) {
    sc = s[index] & 63u;
    mn = s[index + 4] & 63u;
  } else {
    sc = (s[index + 4] & 0x0fu) | ((s[index - 4] >> 6) << 4);
    mn = (s[index + 4] >> 4) | ((s[index] >> 6) << 4);
  }
}

constexpr int kMaxDevices = 64;

// Raise a kernel's dynamic shared memory limit to `bytes` on the current
// device, once: function attributes belong to a device, so `cache[d]` keeps the
// limit set so far on device d (a process may drive several devices).
template <typename F>
inline cudaError_t raise_smem_limit(F kernel, uint32_t bytes, std::atomic<uint32_t>* cache) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
  if (cache[dev].load(std::memory_order_relaxed) >= bytes) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
  if (e == cudaSuccess) cache[dev].store(bytes, std::memory_order_relaxed);
  return e;
}

__host__ __device__ constexpr uint32_t block_bytes_of(uint32_t type) {
  return type == SI_GGML_TYPE_Q4_K ? 144u
         : type == SI_GGML_TYPE_Q5_K ? 176u
         : type == SI_GGML_TYPE_Q6_K ? 210u
                                     : 0u;
}

}  // namespace si
