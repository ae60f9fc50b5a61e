// Per-sequence prologue of a batched GEMM op: the decode path's
// GEMV prologue (RMSNorm / DYNQ8 / gated attention, f5_gemv_core.cuh) for
// one sequence, written as the GEMM's B operand: x8 in the even/odd-permuted
// order of each 8-element block, 128-byte-swizzled K-major rows
// [group][Bp][128] (row b of group g at g * Bp * 128 + swizzle(b, byte)).
#pragma once
#include "f5_batch.cuh"
#include "f5_gemv_core.cuh"
#include "f5_tc.cuh"

namespace f5 {

// xs: shared buffer of (K / 1024) * 4 * 32 uint2 (put8i layout)
template <int MAXB, class SY>
F5_DEV void bprep_seq(const SY &sy, const BprepArgs &pa, int b, uint2 *xs, long long *red, long long *s_r,
                      int *s_meta) {
  const int tid = sy.tid(), BT = sy.n();
  const int nblk = pa.K >> 3;
  if (pa.pro.mode == PRO_X8) {
    const int8_t *x8 = pa.x8_in + (size_t)b * pa.K;
    for (int bb = tid; bb < nblk; bb += BT) {
      const uint2 v = *reinterpret_cast<const uint2 *>(x8 + 8 * bb);
      xs[(((bb >> 7) << 2) + (bb & 3)) * 32 + ((bb >> 2) & 31)] =
          make_uint2(__byte_perm(v.x, v.y, 0x6420), __byte_perm(v.x, v.y, 0x7531));
    }
    if (tid == 0) {
      s_meta[0] = pa.xmeta_in ? pa.xmeta_in[2 * b] : 0;
      s_meta[1] = pa.xmeta_in ? pa.xmeta_in[2 * b + 1] : 0;
    }
  } else {
    // members set one by one (the argument structs are never copied and then
    // modified: see k_dn_step)
    GemvArgs ga;
    ga.K = pa.K;
    ga.err = pa.err;
    ga.abort_flag = nullptr;
    ga.pro.tag_op1 = 0;
    ga.pro.mode = pa.pro.mode;
    ga.pro.src = static_cast<const uint8_t *>(pa.pro.src) + b * pa.src_bs;
    ga.pro.src2 = pa.pro.src2 ? static_cast<const uint8_t *>(pa.pro.src2) + b * pa.src2_bs : nullptr;
    ga.pro.w = pa.pro.w;
    ga.pro.in_f = pa.pro.in_f;
    ga.pro.one_plus = pa.pro.one_plus;
    ga.pro.xq_out.x8 = nullptr;
    ga.pro.xq_out.meta = nullptr;
    ga.pro.dbg = pa.pro.dbg ? pa.pro.dbg + b : nullptr;
    prologue<MAXB>(sy, ga, xs, red, s_r, s_meta);
  }
  sy.sync();
  if (tid == 0) {
    pa.xmeta[2 * b] = s_meta[0];
    pa.xmeta[2 * b + 1] = s_meta[1];
  }
  // 8-element block bb = bytes [8bb, 8bb+8) of the permuted row: group bb/16,
  // 16-byte chunk (bb%16)/2 of the group's 128-byte swizzled row b
  for (int bb = tid; bb < nblk; bb += BT) {
    const uint2 v = xs[(((bb >> 7) << 2) + (bb & 3)) * 32 + ((bb >> 2) & 31)];
    const int g = bb >> 4;
    *reinterpret_cast<uint2 *>(pa.xt + (size_t)g * pa.Bp * 128 + sw128_off(b, (bb & 15) * 8)) = v;
  }
}

}  // namespace f5
