// mbarrier + bulk-copy (TMA, non-tensor) helpers for sm_100a kernels.
// Every bulk copy here is a plain CTA-local copy (one destination CTA).
#pragma once
#include "f5_int.cuh"

namespace f5 {

// ---------------------------------------------------------------------------
// mbarrier / bulk-copy helpers (PTX ISA 8.x, sm_90+; single-destination copies only)
// ---------------------------------------------------------------------------
F5_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
F5_DEV void mbar_init(uint64_t *b, int cnt) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(cnt) : "memory");
}
F5_DEV void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
               : "memory");
}
F5_DEV void mbar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
F5_DEV void mbar_arrive_cnt(uint64_t *b, uint32_t cnt) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(cnt) : "memory");
}
F5_DEV unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#ifndef F5_MBAR_SLEEP_NS
#define F5_MBAR_SLEEP_NS 0
#endif
// Bounded wait on an mbarrier phase: gives up after ~`limit_ns` (the
// caller then records DERR_TIMEOUT and unwinds; nothing ever spins forever).
F5_DEV bool mbar_wait(uint64_t *b, uint32_t parity, unsigned long long limit_ns) {
  const uint32_t addr = smem_u32(b);
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
#if F5_MBAR_SLEEP_NS
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok) : "r"(addr), "r"(parity), "r"((uint32_t)F5_MBAR_SLEEP_NS) : "memory");
#else
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
#endif
    if (ok) return true;
#ifdef F5_MBAR_BACKOFF_NS
    if (it >= 4) __nanosleep(F5_MBAR_BACKOFF_NS);
#endif
    if ((it & 63) == 0) {
      const unsigned long long t = gtimer();
      if (t0 == 0) t0 = t;
      else if (t - t0 > limit_ns) return false;
    }
  }
}
F5_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// L2 eviction priority of the weight stream.  The 4.09 GB of weights of a
// step pass through the 126 MB L2 once per step and are never re-read within
// it: their copies carry evict_first, so they stop displacing the data the
// step reads back (activations, DeltaNet states, conv windows, K/V caches,
// gains), which then stays L2-resident across steps (measured on B200: the
// persistent step 1.646 -> 1.484 ms; an additional evict_last on the state
// and cache copies measured no further change).
F5_DEV uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
F5_DEV void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
               : "memory");
}
// a weight-stream copy
F5_DEV void bulk_g2s_stream(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  bulk_g2s_hint(dst, src, bytes, bar, l2_evict_first());
}

// bring [src, src + bytes) into L2 (16-byte aligned address and size)
F5_DEV void prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 2D tiled tensor copy (box of the tensor map at element coordinates x, y;
// x * element size must be a multiple of 16 bytes), single destination
F5_DEV void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// tma_load_2d of weight-stream tiles (L2 evict_first, see l2_evict_first)
F5_DEV void tma_load_2d_stream(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar)),
        "l"(l2_evict_first())
      : "memory");
}

}  // namespace f5
