// Asynchronous-copy helpers for sm_100a: shared-memory mbarriers, 1-D bulk
// copies global -> shared through the TMA unit (cp.async.bulk, each CTA
// fetching its own data), and bounded waits.
//
// Every wait is bounded: after kSpinLimit polls or 2 s it records an error
// code in this translation unit's device word g_device_error (read through
// mr_device_error_status()) and returns, so a kernel can never spin forever;
// once the word is set, later waits give up at once (see mbar_wait_ns).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mr {

// Device-side error word of this translation unit (first error wins).
// 1 = an mbarrier wait timed out.
static __device__ int g_device_error = 0;

// Host side: read (and optionally clear) this translation unit's word.
// Synchronous; for diagnostics and tests only.
static inline int read_device_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_device_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

constexpr uint32_t kSpinLimit = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
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

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity to complete: gives up
// after kSpinLimit polls or `limit_ns` of wall time, whichever comes first,
// and records the timeout in g_device_error. Once that word is set (by any
// wait of this translation unit, in this launch or an earlier one not yet
// cleared by the host), every later wait that does not complete within 256
// polls gives up at once: a kernel whose copies stopped arriving ends in
// about one time limit instead of one limit per remaining wait, and its
// results are void until the host reads and clears the word.
__device__ __forceinline__ bool mbar_wait_ns(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (*reinterpret_cast<volatile int*>(&g_device_error) != 0) return false;
      if (globaltimer_ns() - t0 > limit_ns) break;
    }
  }
  atomicCAS(&g_device_error, 0, 1);
  return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait_ns(bar, parity, 2000000000ull);
}

// 1-D bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// from global to this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace mr
