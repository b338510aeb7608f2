// Bulk (TMA) copies global -> shared completing on an mbarrier, with a
// bounded wait: a copy that never lands is reported through an error word
// instead of hanging the kernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mb {

__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned phase) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

constexpr int kWaitSpins = 1 << 22;
constexpr int kErrFlagTimeout = 1;
constexpr int kErrFlagBounds = 2;

// Bounded wait on an mbarrier phase; true when it completed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned phase) {
  bool ready = false;
  for (int i = 0; i < kWaitSpins && !ready; ++i) ready = mbar_try_wait(bar, phase);
  return ready;
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) writes into the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

}  // namespace mb
