// Thin wrappers over the sm_90+/sm_100a PTX the GEMV pipeline uses:
// mbarriers (with bounded waits), bulk asynchronous copies global -> shared
// through the TMA engine, and named barriers.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace cw {

// ---- mbarrier ----
CW_DEV void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
CW_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
CW_DEV void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
CW_DEV void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
CW_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
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
CW_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait for the phase of `parity` to complete.  Gives up (returns
// false) after MBAR_TIMEOUT_NS of wall time -- far beyond any legitimate
// wait -- or as soon as another thread of the CTA raised *abort.
constexpr uint64_t MBAR_TIMEOUT_NS = 2000000000ull;
CW_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, const volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; it++) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if ((it & 255u) == 0 && globaltimer_ns() - t0 > MBAR_TIMEOUT_NS) return false;
  }
}

// ---- bulk async copy global -> shared (TMA engine), completes on an mbarrier.
// dst, src 16-byte aligned; bytes a multiple of 16.
CW_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Named barrier over `n` threads (id 1..15; 0 is __syncthreads).
CW_DEV void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

}  // namespace cw
