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
// Time bound for the spin-waits, in SM clock cycles: %clock64 is read in a
// few cycles, whereas a %globaltimer read takes a fraction of a microsecond,
// which a wait loop that reads it on its first miss pays on every stage.
// 4e9 cycles is ~2 s at the 1965 MHz maximum clock -- far beyond any
// legitimate wait -- and proportionally longer at lower clocks.
constexpr long long SPIN_TIMEOUT_CYCLES = 4000000000ll;
CW_DEV long long cycles_now() { return clock64(); }
CW_DEV bool spin_expired(long long t0) { return clock64() - t0 > SPIN_TIMEOUT_CYCLES; }
// Bounded wait for the phase of `parity` to complete.  Gives up (returns
// false) after SPIN_TIMEOUT_CYCLES or as soon as another thread of the CTA
// raised *abort.
CW_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, const volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = cycles_now();
  for (uint32_t it = 1;; it++) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if ((it & 63u) == 0 && spin_expired(t0)) return false;
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
