// tma.cuh — 1-D bulk copies (cp.async.bulk, the TMA engine) into shared
// memory, completed on an mbarrier, with bounded waits.
//
// Every copy reads this GPU's own memory into the issuing CTA's own shared
// memory. Sources and destinations are 16-byte aligned
// and sizes are multiples of 16 bytes (checked by the callers' layouts).
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace chalot {

CHALOT_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// One-shot barrier: init to one arrival, then expect_tx + copies, then wait
// on parity 0.
CHALOT_DEV void mbar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

CHALOT_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Global -> this CTA's shared memory, `bytes` % 16 == 0, both 16-B aligned.
CHALOT_DEV void tma_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy for data read once per step (weights, KV pages): evict first, so
// the streamed bytes do not push the step's small working set (activations,
// routing, tables) and the kernels' code out of L2.
CHALOT_DEV uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// tma_load with an L2 cache policy (l2_evict_first()).
CHALOT_DEV void tma_load_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
      "[%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Waits for phase `parity` of `bar` to complete. Gives up after a bounded
// number of polls (each poll suspends the thread for a hardware-defined
// interval), records the failure in *err and returns false.
CHALOT_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err) {
  const uint32_t a = smem_u32(bar);
  for (int i = 0; i < (1 << 22); ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  if (err) *(volatile unsigned*)err = 1u;  // word 0: a timeout (devstat.h; engine error words)
  return false;
}

}  // namespace chalot
