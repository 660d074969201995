// mbarrier and bulk-copy helpers (inline PTX) shared by the TMA tile kernels
// (tiled_tma.cuh) and the shared-memory look-back scan (scan.cu).
//
// Every wait on an mbarrier is bounded: after 2 s by the global timer (or
// 2^26 polls) the wait gives up and the caller reports it, so a copy that
// never lands cannot hang the GPU.
#pragma once
#include <stdint.h>
#include "common.cuh"

namespace mpb {

MPB_D uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

MPB_D void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

MPB_D void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

MPB_D bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

MPB_D unsigned long long tma_now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for a stage: false after 2 s (or 2^26 polls).
MPB_D bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = tma_now_ns();
  for (long long it = 0; it < (1ll << 26); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (tma_now_ns() - t0 > 2000000000ull) return false;
  }
  return false;
}

// 1-D bulk copy global -> shared on the stage's mbarrier (both addresses
// 16-byte aligned, size a multiple of 16; host-checked). No multicast.
MPB_D void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}


}  // namespace mpb
