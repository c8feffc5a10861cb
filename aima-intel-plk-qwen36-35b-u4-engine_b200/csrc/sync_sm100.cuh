// sync_sm100.cuh — the one copy of the sm_100a synchronisation and bulk-copy
// wrappers every kernel family uses: mbarriers with bounded waits, the global
// nanosecond timer, 1-D bulk copies (cp.async.bulk, no multicast) and the
// generic->async proxy fence. The weight-streaming GEMV, the tcgen05 GEMMs and
// attention, and the fused MoE decode layer all include it.
#pragma once

#include <stdint.h>

namespace iq36 {

// Polls before a bounded wait gives up even if the timer has not run out.
constexpr uint32_t kSpinLimit = 1u << 26;
// Every legitimate wait in this library lasts microseconds; 200 ms means the
// producer or a peer CTA is gone.
constexpr uint64_t kWaitLimitNs = 200000000ull;

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(tx)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
  return t;
}
// Bounded wait on an mbarrier phase: false once kWaitLimitNs have passed or
// after kSpinLimit polls, whichever comes first.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
  return false;
}
// 1-D bulk copy global -> shared of this CTA, completion counted on `bar`
// (bytes). Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
// Order this thread's generic shared-memory accesses before later async-proxy
// (bulk copy / TMA) writes into the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

}  // namespace iq36
