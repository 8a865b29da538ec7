// Tensor Memory Accelerator bulk copies and mbarriers for sm_100a (inline PTX).
//
// Only the 1-D (untiled) form is used: cp.async.bulk global -> shared of a
// whole row, 16-byte aligned source and destination and a size that is a
// multiple of 16 bytes, completing as transaction bytes on an mbarrier of the
// issuing CTA.  No multicast: every copy lands in the issuing CTA's own
// shared memory only.
//
// Every wait is bounded: mbar_wait_bounded gives up after kWaitLimitNs of
// global time (and a fixed number of polls), so a copy that never completes
// cannot hang the GPU; the caller reports the give-up through an error counter
// the host reads (hprn_wait_timeouts).
#pragma once

#include <stdint.h>

namespace hprn {

constexpr uint64_t kWaitLimitNs = 1000000000ull;  // one second per wait
constexpr uint32_t kWaitMaxPolls = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes initialised mbarriers visible to the async proxy (the bulk copies'
// complete_tx) before any copy names them.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy accesses to shared memory before
// later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One arrival that also raises the phase's expected transaction bytes.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// `bytes` from global `src` into this CTA's shared memory at `dst`; completes
// as transaction bytes on `bar`.  L2 policy `pol` (evict_first for streamed rows).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for phase `parity` of `bar` to complete; false if it did not within
// `limit_ns` of global time (or kWaitMaxPolls polls).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kWaitMaxPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) break;
  }
  return false;
}

// Counts `bytes` of the current phase's expected transactions as done, as a
// copy's completion would.  Only the test hook that stalls a staged row uses
// it: to release the bytes that row's phase expected beyond its copies.
__device__ __forceinline__ void mbar_complete_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

}  // namespace hprn
