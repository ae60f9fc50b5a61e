// tcgen05 (5th-generation tensor core) helpers for sm_100a: TMEM allocation,
// shared-memory matrix descriptors, the int8 MMA, its commit to an mbarrier
// and the TMEM -> register loads of the accumulators.
#pragma once
#include "f5_kernels.cuh"
#include "f5_tma.cuh"

namespace f5 {

// K-major operand tile of R rows x 128 bytes in the 128-byte swizzle layout:
// row r at r * 128, 16-byte chunk c stored at chunk c ^ (r & 7); 8-row
// groups 1024 bytes apart (SBO).  The tile must start 1024-byte aligned.
F5_DEV uint32_t sw128_off(int r, int byte) { return (uint32_t)(r * 128 + ((((byte >> 4) ^ r) & 7) << 4) + (byte & 15)); }

// shared-memory matrix descriptor of such a tile at shared address `addr`
// (start >> 4 in bits 0-13, leading offset 1 (unused by swizzled K-major
// tiles), stride offset 1024 >> 4, descriptor version 1 in bits 46-47,
// layout SWIZZLE_128B = 2 in bits 61-63).  Advancing along K by 32 bytes
// inside the 128-byte swizzle row adds 2 to the start field.
F5_DEV uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// K-major operand tile of R rows x 32 bytes without swizzle: 8-row x
// 16-byte core matrices (128 contiguous bytes), the two K halves 128 bytes
// apart (leading offset), 8-row groups 256 bytes apart (stride offset)
F5_DEV uint32_t kn32_off(int r, int byte) { return (uint32_t)((r >> 3) * 256 + (byte >> 4) * 128 + (r & 7) * 16 + (byte & 15)); }
F5_DEV uint64_t kn32_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) | (1ull << 46);
}

// instruction descriptor of kind::i8: D int32 (format 2, bits 4-5), A u8
// (0, bits 7-9), B s8 (1, bits 10-12), both K-major, N >> 3 in bits 17-22,
// M >> 4 in bits 24-28
F5_DEV_HOST_INLINE uint32_t idesc_u8s8(int M, int N) {
  return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// the same with A s8 (format 1)
F5_DEV_HOST_INLINE uint32_t idesc_s8s8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

F5_DEV void tc_alloc(uint32_t *dst_smem, uint32_t ncols) {   // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
F5_DEV void tc_dealloc(uint32_t taddr, uint32_t ncols) {   // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
F5_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
F5_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A * B^T, M x N x 32 bytes of K, one thread
F5_DEV void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// the same with A read from tensor memory: a_tmem holds M rows (lanes) x 32
// bytes of K (8 columns, 4 bytes of K per 32-bit column, little-endian)
F5_DEV void tc_mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// 32 lanes x 32 columns from registers (thread i -> lane base + i)
F5_DEV void tc_st32(uint32_t t, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(t),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
F5_DEV void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// arrive once on `bar` when every MMA this thread issued so far has completed
F5_DEV void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
F5_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x N columns of 32-bit cells: thread i gets lane (base lane + i)
template <int N>
F5_DEV void tc_ld(uint32_t taddr, int32_t (&v)[N]);
template <>
F5_DEV void tc_ld<4>(uint32_t t, int32_t (&v)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(t)
               : "memory");
}
template <>
F5_DEV void tc_ld<8>(uint32_t t, int32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(t)
               : "memory");
}
template <>
F5_DEV void tc_ld<16>(uint32_t t, int32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(t)
      : "memory");
}
template <>
F5_DEV void tc_ld<32>(uint32_t t, int32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(t)
      : "memory");
}

}  // namespace f5
