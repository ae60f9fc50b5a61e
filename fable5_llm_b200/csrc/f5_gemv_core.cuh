// Device core of the W4A8 GEMV, shared by the per-op kernel k_gemv and the
// persistent decode kernel: nibble dot products, the group-scale law, the
// per-CTA prologues that quantize the input vector, and the epilogues.
// The law and the memory layout are described in f5_gemv.cu.
#pragma once
#include <climits>
#include "f5_block.cuh"
#include "f5_kernels.cuh"
#include "f5_tma.cuh"

// optional phase marks inside the prologue (the persistent kernel's trace)
#ifndef F5_PRO_MARK
#define F5_PRO_MARK(k) \
  do {               \
  } while (0)
#endif

namespace f5 {

// ---- dataflow-tagged activation words (see StepParams / mega_epoch) ----
F5_DEV uint32_t mk_tag(uint32_t epoch, int op1) { return (epoch << 8) | ((uint32_t)(op1 - 1) & 0xFFu); }
F5_DEV uint32_t tag_word(uint32_t tag, int32_t v) { return (tag << 16) | ((uint32_t)v & 0xFFFFu); }
F5_DEV int32_t tag_s16(uint32_t w) { return (int32_t)(int16_t)(w & 0xFFFFu); }
// a tagged output word: into this GPU's twin and, row-sharded, every peer's
// (the fused all-gather of the GEMV's output rows: plain 4-byte stores)
F5_DEV void st_tagged(const GemvArgs &a, uint32_t *p, uint32_t w) {
  if (a.nrank <= 1) {
    *p = w;
    return;
  }
  for (int r = 0; r < a.nrank; ++r) *reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(p) + a.peer_delta[r]) = w;
}

// L2 loads the compiler must issue on every call (poll loops re-read them;
// a plain __ldcg could be hoisted out of the loop)
F5_DEV uint4 ld_cg_poll(const uint4 *p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}
F5_DEV uint2 ld_cg_poll(const uint2 *p) {
  uint2 v;
  asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
F5_DEV uint32_t ld_cg_poll(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded poll until the n words at p (n = 1, 2 or 8; 16-byte aligned for 8)
// all carry `tag`; reads at L2.  Gives up after 1 s (or once the kernel's
// abort flag is up, polled every ~20 us), then raises DERR_TIMEOUT and the
// abort flag; the caller carries on with whatever it read.
template <int N>
F5_DEV bool ld_tagged(const uint32_t *p, uint32_t tag, uint32_t (&w)[N], unsigned *abortf, uint32_t *err) {
  unsigned long long t0 = 0, tpoll = 0;
  for (uint32_t it = 0;; ++it) {
    if (N == 8) {
      const uint4 a = ld_cg_poll(reinterpret_cast<const uint4 *>(p)), b = ld_cg_poll(reinterpret_cast<const uint4 *>(p) + 1);
      w[0] = a.x; w[1 % N] = a.y; w[2 % N] = a.z; w[3 % N] = a.w;
      w[4 % N] = b.x; w[5 % N] = b.y; w[6 % N] = b.z; w[7 % N] = b.w;
    } else if (N == 2) {
      const uint2 a = ld_cg_poll(reinterpret_cast<const uint2 *>(p));
      w[0] = a.x; w[1 % N] = a.y;
    } else {
      w[0] = ld_cg_poll(p);
    }
    bool ok = true;
#pragma unroll
    for (int i = 0; i < N; ++i) ok &= (w[i] >> 16) == tag;
    if (ok) return true;
    if ((it & 7) == 7) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t0 == 0) {
        t0 = t;
        tpoll = t + 20000;
      } else if (t >= tpoll) {
        if (abortf && *reinterpret_cast<volatile unsigned *>(abortf)) return false;
        if (t - t0 > 1000000000ull) {
          atomicOr(err, DERR_TIMEOUT);
          if (abortf) atomicExch(abortf, 1u);
          return false;
        }
        tpoll = t + 20000;
      }
    }
  }
}

// ld_tagged over N independent words: every still-pending word is loaded
// in the same round, so a thread waits one L2 round trip per poll instead of
// one per word.  Words with act[i] false are skipped (w[i] = 0).
template <int N>
F5_DEV bool ld_tagged_multi(const uint32_t *const (&p)[N], const bool (&act)[N], uint32_t tag, uint32_t (&w)[N],
                            unsigned *abortf, uint32_t *err) {
  bool done[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    done[i] = !act[i];
    w[i] = 0;
  }
  unsigned long long t0 = 0, tpoll = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t v[N];
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = done[i] ? 0u : ld_cg_poll(p[i]);
    bool ok = true;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      if (!done[i] && (v[i] >> 16) == tag) {
        w[i] = v[i];
        done[i] = true;
      }
      ok &= done[i];
    }
    if (ok) return true;
    if ((it & 7) == 7) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t0 == 0) {
        t0 = t;
        tpoll = t + 20000;
      } else if (t >= tpoll) {
        if (abortf && *reinterpret_cast<volatile unsigned *>(abortf)) return false;
        if (t - t0 > 1000000000ull) {
          atomicOr(err, DERR_TIMEOUT);
          if (abortf) atomicExch(abortf, 1u);
          return false;
        }
        tpoll = t + 20000;
      }
    }
  }
}

// ld_tagged over MAXB 8-word blocks (block j at p[j], 16-byte aligned):
// all blocks are loaded in the same round, so a thread waits one L2 round
// trip per poll instead of one per block.  Blocks with act[j]
// false are skipped; raw[j] receives block j's eight int16 values.
template <int MAXB>
F5_DEV bool ld_tagged_blocks(const uint32_t *const (&p)[MAXB], const bool (&act)[MAXB], uint32_t tag,
                             uint4 (&raw)[MAXB], unsigned *abortf, uint32_t *err) {
  unsigned long long t0 = 0, tpoll = 0;
  for (uint32_t it = 0;; ++it) {
    bool ok = true;
#pragma unroll
    for (int j = 0; j < MAXB; ++j) {
      const uint4 lo = ld_cg_poll(reinterpret_cast<const uint4 *>(p[j]));
      const uint4 hi = ld_cg_poll(reinterpret_cast<const uint4 *>(p[j]) + 1);
      const uint32_t t8 = ((lo.x >> 16) ^ tag) | ((lo.y >> 16) ^ tag) | ((lo.z >> 16) ^ tag) | ((lo.w >> 16) ^ tag) |
                          ((hi.x >> 16) ^ tag) | ((hi.y >> 16) ^ tag) | ((hi.z >> 16) ^ tag) | ((hi.w >> 16) ^ tag);
      ok &= !act[j] || t8 == 0u;
      raw[j] = act[j] ? make_uint4((lo.x & 0xFFFFu) | (lo.y << 16), (lo.z & 0xFFFFu) | (lo.w << 16),
                                   (hi.x & 0xFFFFu) | (hi.y << 16), (hi.z & 0xFFFFu) | (hi.w << 16))
                      : make_uint4(0, 0, 0, 0);
    }
    if (ok) return true;
    // back off between rounds: every CTA polling all its blocks at full rate
    // floods L2 with loads of the lines the last writers are storing to
    __nanosleep(100);
    if ((it & 7) == 7) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t0 == 0) {
        t0 = t;
        tpoll = t + 20000;
      } else if (t >= tpoll) {
        if (abortf && *reinterpret_cast<volatile unsigned *>(abortf)) return false;
        if (t - t0 > 1000000000ull) {
          atomicOr(err, DERR_TIMEOUT);
          if (abortf) atomicExch(abortf, 1u);
          return false;
        }
        tpoll = t + 20000;
      }
    }
  }
}

F5_DEV uint4 ld_stream16(const uint8_t *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
F5_DEV uint32_t ld_u16(const uint8_t *p) {
  unsigned short v;
  asm("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

F5_DEV int dot_word(uint32_t w, uint2 x, int acc) {
  acc = __dp4a((int)((w << 4) & 0xF0F0F0F0u), (int)x.x, acc);
  acc = __dp4a((int)(w & 0xF0F0F0F0u), (int)x.y, acc);
  return acc;
}
F5_DEV int dot32(uint4 w, uint2 x0, uint2 x1, uint2 x2, uint2 x3) {
  int acc = dot_word(w.x, x0, 0);
  acc = dot_word(w.y, x1, acc);
  acc = dot_word(w.z, x2, acc);
  acc = dot_word(w.w, x3, acc);
  return acc;   // 16 * sum(w*x) over 32 weights, |.| < 2^20
}

F5_DEV unsigned long long argmax_key(int32_t y, int row) {
  return ((unsigned long long)((uint32_t)y ^ 0x80000000u) << 32) |
         (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}

// y32 for one row from the lane-reduced p16 (= 16 p)
F5_DEV int32_t finish_y32(long long p16, int sh, uint32_t *err, long long *p_exact) {
  const long long p = p16 >> 4;
  const long long y = rshr(p, sh);
  if (y >= (1ll << 31) || y <= -(1ll << 31)) atomicOr(err, DERR_Y32_OVERFLOW);
  if (p_exact) *p_exact = p;
  return (int32_t)y;
}

F5_DEV void load8_i16(const int16_t *p, long long v[8]) {
  const uint4 u = *reinterpret_cast<const uint4 *>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = (int16_t)(w[j] & 0xFFFFu);
    v[2 * j + 1] = (int16_t)(w[j] >> 16);
  }
}
F5_DEV void load8_i64(const int64_t *p, long long v[8]) {
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    const longlong2 u = __ldcg(reinterpret_cast<const longlong2 *>(p + j));
    v[j] = u.x;
    v[j + 1] = u.y;
  }
}
F5_DEV void put8(uint2 *xs, int b, const long long x[8]) {
  uint32_t ev = 0, od = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    ev |= ((uint32_t)(x[2 * j] & 0xFF)) << (8 * j);
    od |= ((uint32_t)(x[2 * j + 1] & 0xFF)) << (8 * j);
  }
  xs[(((b >> 7) << 2) + (b & 3)) * 32 + ((b >> 2) & 31)] = make_uint2(ev, od);
}

// rmsnorm_fx element (ref/layer_fixed.py:1242-1278): clip16(rshr(clip33(
// rshr(x*r, 30-e)) * gain, 14)).  Fast form for the prologue: x is int16,
// 0 < r < 2^31 (rsqrt_q), s = 30 - e >= 1 and |gain| < 2^31.  Clamping the
// intermediate to int32 instead of 33 bits is exact: any |y| >= 2^31 with a
// nonzero gain gives |y * gain| >= 2^31, which clip16 saturates either way
// with the same sign (gain 0 gives 0 either way).
F5_DEV long long rms_elem(long long x, long long r, int e, long long gain) {
  long long y = rshr(x * r, 30 - e);
  y = clip(y, -(1ll << 32), (1ll << 32) - 1);
  return clip16(rshr(y * gain, 14));
}
F5_DEV int32_t rms_elem32(int32_t x, int32_t r, int s, int32_t gain) {
  const long long v = (long long)x * r;                        // |v| < 2^46
  const unsigned long long av = (unsigned long long)(v < 0 ? -v : v);
  const unsigned long long q = (av + (1ull << (s - 1))) >> s;  // rshr of |v|, half away from zero
  const long long yq = q > 0x7FFFFFFFull ? 0x80000000ll : (long long)q;
  const int32_t y = (int32_t)(v < 0 ? (yq > 0x7FFFFFFFll ? INT32_MIN : -(int32_t)yq) : (yq > 0x7FFFFFFFll ? INT32_MAX : (int32_t)yq));
  const long long t = (long long)y * gain;                     // |t| < 2^62
  const unsigned long long at = (unsigned long long)(t < 0 ? -t : t);
  const unsigned long long u = (at + 8192) >> 14;
  const long long c = u > 32768ull ? 32768 : (long long)u;
  return (int32_t)(t < 0 ? -c : (c > 32767 ? 32767 : c));
}

// rms_elem32 for 17 <= s <= 47 (every int16 RMSNorm input: s = 30 - e of
// rsqrt_q is >= 17 for any sum of squares >= 1) in 32-bit integer
// arithmetic.  With r = rh 2^16 + rl (0 < r < 2^31, rh < 2^15):
//   vh = |x| rh + ((|x| rl) >> 16) = floor(|x| r / 2^16)  (< 2^31),
//   q  = (vh + 2^(s-17)) >> (s-16) = rshr(|x| r, s)        (< 2^31, no clamp),
// exact because 2^(s-1) is a multiple of 2^16 (nested floor division); the
// gain product |t| = q |gain| saturates clip16 once it reaches 2^29 - 8192,
// so only its high word's zero test and the low word are needed.
F5_DEV int32_t rms_elem_s17(int32_t x, uint32_t rh, uint32_t rl, int s, int32_t gain) {
  const uint32_t ax = (uint32_t)(x < 0 ? -x : x);
  const uint32_t vh = ax * rh + ((ax * rl) >> 16);
  const uint32_t q = (vh + (1u << (s - 17))) >> (s - 16);
  const uint32_t ag = gain < 0 ? 0u - (uint32_t)gain : (uint32_t)gain;
  const uint32_t lo = q * ag, hi = __umulhi(q, ag);
  const uint32_t c = (hi != 0u || lo >= (1u << 29) - 8192u) ? 32768u : (lo + 8192u) >> 14;
  return ((x < 0) != (gain < 0)) ? -(int32_t)c : (int32_t)(c < 32767u ? c : 32767u);
}

// element j (0..7) of 8 int16 packed in a uint4
F5_DEV long long get16(const uint4 &u, int j) {
  const uint32_t w = (j >> 1) == 0 ? u.x : ((j >> 1) == 1 ? u.y : ((j >> 1) == 2 ? u.z : u.w));
  return (long long)(int16_t)((j & 1) ? (w >> 16) : (w & 0xFFFFu));
}
F5_DEV int32_t get16i(const uint4 &u, int j) {
  const uint32_t w = (j >> 1) == 0 ? u.x : ((j >> 1) == 1 ? u.y : ((j >> 1) == 2 ? u.z : u.w));
  return (int32_t)(int16_t)((j & 1) ? (w >> 16) : (w & 0xFFFFu));
}
// rmsnorm_fx of one 8-element block outside rms_elem_s17's domain (the
// 32-bit law for 1 <= s <= 62, else the 64-bit law).  Kept out of line:
// the decode step never takes it (int16 inputs always give 17 <= s <= 47),
// and as inlined code it only enlarged the persistent kernel's instruction
// footprint (measured 0.6 % of the step).
static __device__ __noinline__ uint4 rms_block_slow(uint4 raw, int4 w0, int4 w1, long long r, int e, int add1) {
  const int wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const bool fast = r > 0 && r < (1ll << 31) && 30 - e >= 1 && 30 - e <= 62;
  uint32_t pk[4];
  for (int k = 0; k < 8; k += 2) {
    int32_t x0, x1;
    if (fast) {
      x0 = rms_elem32(get16i(raw, k), (int32_t)r, 30 - e, wv[k] + add1);
      x1 = rms_elem32(get16i(raw, k + 1), (int32_t)r, 30 - e, wv[k + 1] + add1);
    } else {
      x0 = (int32_t)rms_elem(get16(raw, k), r, e, (long long)wv[k] + add1);
      x1 = (int32_t)rms_elem(get16(raw, k + 1), r, e, (long long)wv[k + 1] + add1);
    }
    pk[k >> 1] = ((uint32_t)x0 & 0xFFFFu) | ((uint32_t)x1 << 16);
  }
  return make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// the int8 values q[0..7] of block b into the lane-major even/odd layout
F5_DEV void put8i(uint2 *xs, int b, const int32_t q[8]) {
  const uint32_t ev = __byte_perm(__byte_perm(q[0], q[2], 0x0040), __byte_perm(q[4], q[6], 0x0040), 0x5410);
  const uint32_t od = __byte_perm(__byte_perm(q[1], q[3], 0x0040), __byte_perm(q[5], q[7], 0x0040), 0x5410);
  xs[(((b >> 7) << 2) + (b & 3)) * 32 + ((b >> 2) & 31)] = make_uint2(ev, od);
}

F5_DEV int seg_of(const GemvArgs &a, int u) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < GEMV_MAX_SEG; ++i)
    if (i < a.nseg && u >= a.seg[i].unit_begin) s = i;
  return s;
}

// Deterministic chunking of this CTA's unit range (same in producer and
// consumers): a chunk is <= R rows of ONE segment (paired: R/2 row pairs).
struct Chunk {
  int seg, r0, n, u;
};
F5_DEV bool next_chunk(const GemvArgs &a, int &u, int u1, Chunk &ch) {
  if (u >= u1) return false;
  const int s = seg_of(a, u);
  const GemvSeg &sg = a.seg[s];
  const int seg_end = (s + 1 < a.nseg) ? a.seg[s + 1].unit_begin : a.total_units;
  const int ru = sg.mode == GM_SILU_MUL ? (a.rows_per_stage >> 1) : a.rows_per_stage;
  const int n = min(min(ru, u1 - u), seg_end - u);
  ch.seg = s;
  ch.r0 = u - sg.unit_begin;
  ch.n = n;
  ch.u = u;
  u += n;
  return true;
}

// 16*sum_k w*x over one row held in shared memory (lane-strided 16 B reads)
template <int NCH>
F5_DEV long long row_dot(const uint8_t *row, int K2, int gshift, int lane, const uint2 (&xr)[4][4],
                         const uint2 *xs) {
  long long acc = 0;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int boff = c * 512 + lane * 16;
    if (boff < K2) {
      const uint4 w = *reinterpret_cast<const uint4 *>(row + boff);
      const uint32_t m = *reinterpret_cast<const uint16_t *>(row + K2 + 2 * (boff >> gshift));
      int d;
      if (NCH <= 4) {
        d = dot32(w, xr[c & 3][0], xr[c & 3][1], xr[c & 3][2], xr[c & 3][3]);
      } else {
        const uint2 *x = xs + (c << 2) * 32 + lane;
        d = dot32(w, x[0], x[32], x[64], x[96]);
      }
      acc += (long long)m * d;
    }
  }
  return acc;
}

F5_DEV long long warp_sum_ll(long long v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Exact warp sum of a row's per-lane partials p (|p| < 2^39: at most twelve
// group terms m * d with m < 2^16, |d| < 2^19) with two 32-bit redux.sync
// adds instead of a 64-bit shuffle tree: p = hi * 2^22 + lo with
// lo = p mod 2^22 in [0, 2^22) and hi = floor(p / 2^22), |hi| < 2^17, so
// sum(lo) < 2^27 and |sum(hi)| < 2^22 both fit 32 bits.
F5_DEV long long warp_sum_row(long long p) {
  const unsigned lo = (unsigned)p & 0x3FFFFFu;
  const int hi = (int)(p >> 22);
  const unsigned slo = __reduce_add_sync(0xffffffffu, lo);
  const int shi = __reduce_add_sync(0xffffffffu, hi);
  return ((long long)shi << 22) + (long long)slo;
}

// 16*sum_k w*x over one K=4096 row held in shared memory, x held in
// registers (lane l owns bytes [c*512 + 16l, +16) of the weights, c < 4)
F5_DEV long long row_dot4096(const uint8_t *row, int lane, const uint2 (&xr)[4][4]) {
  long long acc = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int boff = c * 512 + lane * 16;
    const uint4 w = *reinterpret_cast<const uint4 *>(row + boff);
    const uint32_t m = *reinterpret_cast<const uint16_t *>(row + 2048 + 2 * (boff >> 6));
    acc += (long long)m * dot32(w, xr[c][0], xr[c][1], xr[c][2], xr[c][3]);
  }
  return acc;
}


// two K = 4096 rows at once: independent chains the scheduler interleaves
F5_DEV void row_dot4096x2(const uint8_t *row0, const uint8_t *row1, int lane, const uint2 (&xr)[4][4],
                          long long &out0, long long &out1) {
  long long a0 = 0, a1 = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int boff = c * 512 + lane * 16;
    const uint4 w0 = *reinterpret_cast<const uint4 *>(row0 + boff);
    const uint4 w1 = *reinterpret_cast<const uint4 *>(row1 + boff);
    const uint32_t m0 = *reinterpret_cast<const uint16_t *>(row0 + 2048 + 2 * (boff >> 6));
    const uint32_t m1 = *reinterpret_cast<const uint16_t *>(row1 + 2048 + 2 * (boff >> 6));
    a0 += (long long)m0 * dot32(w0, xr[c][0], xr[c][1], xr[c][2], xr[c][3]);
    a1 += (long long)m1 * dot32(w1, xr[c][0], xr[c][1], xr[c][2], xr[c][3]);
  }
  out0 = a0;
  out1 = a1;
}

// Redundant per-CTA computation of the GEMV's quantized input (see GemvPro).
// Every value is read from global memory once and held in registers across
// the reduction passes (MAXB 8-element blocks per thread).
// `epoch` != 0 with P.tag_op1 != 0: the input vector is dataflow-tagged
// (persistent kernel) and each thread polls its words until they are ready.
template <int MAXB, class SY>
F5_DEV void prologue(const SY &sy, const GemvArgs &a, uint2 *xs, long long *red, long long *s_r, int *s_meta,
                     uint32_t epoch = 0, const int32_t *gains_smem = nullptr) {
  const int tid = sy.tid(), BT = sy.n(), K = a.K, nblk = K >> 3;
  const GemvPrologue &P = a.pro;
  const bool store = (P.xq_out.x8 != nullptr) && blockIdx.x == 0;
  const uint32_t in_tag = (epoch && P.tag_op1) ? mk_tag(epoch, P.tag_op1) : 0u;
  long long q[8];
  if (P.mode == PRO_RMSNORM || P.mode == PRO_DYNQ8) {
    const int16_t *src = static_cast<const int16_t *>(P.src);
    uint4 raw[MAXB];
    if (in_tag && MAXB > 1) {   // several blocks per thread: polled together
      const uint32_t *pb[MAXB];
      bool act[MAXB];
#pragma unroll
      for (int j = 0; j < MAXB; ++j) {
        const int b = tid + j * BT;
        act[j] = b < nblk;
        pb[j] = static_cast<const uint32_t *>(P.src) + 8 * (act[j] ? b : 0);
      }
      ld_tagged_blocks<MAXB>(pb, act, in_tag, raw, a.abort_flag, a.err);
    } else if (in_tag) {
#pragma unroll
      for (int j = 0; j < MAXB; ++j) {
        const int b = tid + j * BT;
        uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (b < nblk) ld_tagged<8>(static_cast<const uint32_t *>(P.src) + 8 * b, in_tag, w, a.abort_flag, a.err);
        raw[j] = make_uint4((w[0] & 0xFFFFu) | (w[1] << 16), (w[2] & 0xFFFFu) | (w[3] << 16),
                            (w[4] & 0xFFFFu) | (w[5] << 16), (w[6] & 0xFFFFu) | (w[7] << 16));
      }
    } else {
#pragma unroll
      for (int j = 0; j < MAXB; ++j) {
        const int b = tid + j * BT;
        raw[j] = b < nblk ? __ldcg(reinterpret_cast<const uint4 *>(src + 8 * b)) : make_uint4(0, 0, 0, 0);
      }
    }
    if constexpr (MAXB <= 2) {
      if (P.mode == PRO_RMSNORM) {     // ref/layer_fixed.py:1242-1278 (H = 4096)
        int4 wl[MAXB][2];
#pragma unroll
        for (int j = 0; j < MAXB; ++j) {
          const int b = tid + j * BT;
          // gains from the caller's shared-memory copy, else streamed at L2 (__ldcg)
          const int32_t *gw = gains_smem ? gains_smem : P.w;
          if (b >= nblk) {
            wl[j][0] = wl[j][1] = make_int4(0, 0, 0, 0);
          } else if (gains_smem) {
            wl[j][0] = *reinterpret_cast<const int4 *>(gw + 8 * b);
            wl[j][1] = *reinterpret_cast<const int4 *>(gw + 8 * b + 4);
          } else {
            wl[j][0] = __ldcg(reinterpret_cast<const int4 *>(gw + 8 * b));
            wl[j][1] = __ldcg(reinterpret_cast<const int4 *>(gw + 8 * b + 4));
          }
        }
        long long ss = 0;   // < 16 * 2^30 per thread
#pragma unroll
        for (int j = 0; j < MAXB; ++j)
#pragma unroll
          for (int k = 0; k < 8; ++k) { const int32_t v = get16i(raw[j], k); ss += (long long)(v * v); }
        ss = g_sum_split(sy, ss, red);   // the same value in every thread
        F5_PRO_MARK(4);
        // every thread evaluates rsqrt_q itself (uniform input: the LUT read
        // is a broadcast) instead of one thread and a barrier to publish it
        int64_t r;
        int e;
        rsqrt_q((uint64_t)(ss == 0 ? 1 : ss), 2 * P.in_f + (31 - __clz(K)), r, e);
        F5_PRO_MARK(6);
        const int add1 = P.one_plus ? (1 << 14) : 0;
        // fast path when rsqrt's r and shift are in rms_elem32's domain (always
        // for int16 inputs of H = 4096); the general law otherwise
        const bool fast17 = r > 0 && r < (1ll << 31) && 30 - e >= 17 && 30 - e <= 47;
        const uint32_t rh = (uint32_t)r >> 16, rl = (uint32_t)r & 0xFFFFu;
#pragma unroll
        for (int j = 0; j < MAXB; ++j) {
          if (!fast17) {
            raw[j] = rms_block_slow(raw[j], wl[j][0], wl[j][1], r, e, add1);
            continue;
          }
          const int wv[8] = {wl[j][0].x, wl[j][0].y, wl[j][0].z, wl[j][0].w,
                             wl[j][1].x, wl[j][1].y, wl[j][1].z, wl[j][1].w};
          uint32_t pk[4];
#pragma unroll
          for (int k = 0; k < 8; k += 2) {
            const int32_t x0 = rms_elem_s17(get16i(raw[j], k), rh, rl, 30 - e, wv[k] + add1);
            const int32_t x1 = rms_elem_s17(get16i(raw[j], k + 1), rh, rl, 30 - e, wv[k + 1] + add1);
            pk[k >> 1] = ((uint32_t)x0 & 0xFFFFu) | ((uint32_t)x1 << 16);
          }
          raw[j] = make_uint4(pk[0], pk[1], pk[2], pk[3]);   // normalised, int16
        }
      }
    } else {
      if (P.mode == PRO_RMSNORM && tid == 0) atomicOr(a.err, DERR_RANGE);   // RMSNorm is bound to K <= 4096
    }
    unsigned mx = 0;   // int16 magnitudes: 32-bit max
#pragma unroll
    for (int j = 0; j < MAXB; ++j)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int32_t v = get16i(raw[j], k);
        const unsigned m = (unsigned)(v < 0 ? -v : v);
        mx = m > mx ? m : mx;
      }
    mx = g_max_u32(sy, mx, red);
    F5_PRO_MARK(5);
    const int ex = dynq8_e(mx);
#pragma unroll
    for (int j = 0; j < MAXB; ++j) {
      const int b = tid + j * BT;
      if (b < nblk) {
        int32_t qi[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          qi[k] = dynq8_apply32(get16i(raw[j], k), ex);
          if (store) P.xq_out.x8[8 * b + k] = (int8_t)qi[k];
        }
        put8i(xs, b, qi);
      }
    }
    if (tid == 0) { s_meta[0] = ex; s_meta[1] = P.in_f; }
  } else if constexpr (MAXB <= 2) {  // PRO_ATTN_GATE / _ACC (ref/layer_fixed.py:1436-1449); K = NQ*HD = 4096
    long long v[MAXB][8];
#pragma unroll
    for (int j = 0; j < MAXB; ++j) {
      const int b = tid + j * BT;
      if (b >= nblk) {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[j][k] = 0;
      } else if (P.mode == PRO_ATTN_GATE) {
        load8_i64(static_cast<const int64_t *>(P.src) + 8 * b, v[j]);
      } else {
        // og = sigmoid_q(rshr(gate, QKV_F - 12)) = sigmoid_q(gate << (12 - QKV_F))
        const int4 a0 = __ldcg(reinterpret_cast<const int4 *>(static_cast<const int32_t *>(P.src) + 8 * b));
        const int4 a1 = __ldcg(reinterpret_cast<const int4 *>(static_cast<const int32_t *>(P.src) + 8 * b + 4));
        const int i0 = 8 * b, hq = i0 >> 8, d0 = i0 & 255;
        uint4 gr;
        if (in_tag) {   // tagged q|gate words (ordered by the grid barrier before this op)
          uint32_t w[8];
          ld_tagged<8>(static_cast<const uint32_t *>(P.src2) + (size_t)hq * 512 + 256 + d0, in_tag, w, a.abort_flag,
                       a.err);
          gr = make_uint4((w[0] & 0xFFFFu) | (w[1] << 16), (w[2] & 0xFFFFu) | (w[3] << 16),
                          (w[4] & 0xFFFFu) | (w[5] << 16), (w[6] & 0xFFFFu) | (w[7] << 16));
        } else {
          gr = __ldcg(reinterpret_cast<const uint4 *>(static_cast<const int16_t *>(P.src2) + (size_t)hq * 512 + 256 + d0));
        }
        const int av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) v[j][k] = (long long)av[k] * sigmoid_q(get16(gr, k) << (12 - QKV_F));
      }
    }
    unsigned long long mx = 0;
#pragma unroll
    for (int j = 0; j < MAXB; ++j)
#pragma unroll
      for (int k = 0; k < 8; ++k) { const unsigned long long m = uabs(v[j][k]); mx = m > mx ? m : mx; }
    F5_PRO_MARK(4);
    mx = g_max_ull(sy, mx, reinterpret_cast<unsigned long long *>(red));
    F5_PRO_MARK(6);
    int ka = bf_shift(mx);
    if (ka < 0) ka = 0;                      // attn_o_shift clamp (ref/layer_fixed.py:489-506)
    unsigned long long mg = 0;
#pragma unroll
    for (int j = 0; j < MAXB; ++j)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        v[j][k] = clip16(rshr(v[j][k], ka));
        const unsigned long long m = uabs(v[j][k]);
        mg = m > mg ? m : mg;
      }
    mg = g_max_ull(sy, mg, reinterpret_cast<unsigned long long *>(red));
    F5_PRO_MARK(5);
    const int ex = dynq8_e(mg);
#pragma unroll
    for (int j = 0; j < MAXB; ++j) {
      const int b = tid + j * BT;
      if (b < nblk) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          q[k] = dynq8_apply(v[j][k], ex);
          if (store) P.xq_out.x8[8 * b + k] = (int8_t)q[k];
        }
        put8(xs, b, q);
      }
    }
    if (tid == 0) {
      s_meta[0] = ex;
      s_meta[1] = QKV_F + GAT_F - ka;
      if (P.dbg && blockIdx.x == 0) *P.dbg = ka;
    }
  } else {
    if (tid == 0) atomicOr(a.err, DERR_RANGE);   // the attention gate prologue is bound to K <= 4096
  }
  if (store && tid == 0) {
    P.xq_out.meta[0] = s_meta[0];
    P.xq_out.meta[1] = s_meta[1];
  }
}

// ---------------------------------------------------------------------------
// Epilogues (ref/layer_fixed.py:1224-1236 matvec_to and its call sites)
// ---------------------------------------------------------------------------
// conv4 + SiLU of one channel (ref/layer_fixed.py:1511-1520): ring word rw
// holds the 4 int16 slots, cw the 4 weights, v this step's pre-conv input
// ring slot k (0..3) of the four int16 slots packed in rw, selected in
// registers (a dynamically indexed local array would live in local memory)
F5_DEV long long ring_slot(uint2 rw, int k) {
  const uint32_t w = (k & 2) ? rw.y : rw.x;
  return (long long)(int16_t)((k & 1) ? (w >> 16) : (w & 0xFFFFu));
}
F5_DEV int32_t conv_silu(long long v, uint2 rw, int4 cw, int T) {
  const long long acc = ring_slot(rw, (T + 1) & 3) * cw.x + ring_slot(rw, (T + 2) & 3) * cw.y +
                        ring_slot(rw, (T + 3) & 3) * cw.z + v * cw.w;
  const long long pre = clip(rshr(acc, RS_F + CW_F - 12), -(1 << 20), (1 << 20) - 1);
  const long long co = clip16(silu_q(pre));
  return (int32_t)rshr(co, 12 - QKV_F);
}
// decay gate of one head (ref/layer_fixed.py:1532-1538)
F5_DEV int32_t decay_gate(long long v, int32_t dt_bias, int32_t A) {
  const long long sp = softplus_q(v + dt_bias);
  const long long g = -rshr((long long)A * sp, 15 + 12 - 16);
  const long long dec = rshr(exp_neg_q(g < 0 ? g : 0), 15);
  return (int32_t)(dec > 32767 ? 32767 : dec);
}
// Per-thread residual statistics of GM_RESID outputs (GemvSeg::rstat),
// folded into the global words once per warp by rstat_flush.
struct RStat {
  unsigned mx = 0u, n = 0u;
  F5_DEV void add(int32_t v) {
    const unsigned m = (unsigned)(v < 0 ? -v : v);
    mx = m > mx ? m : mx;
    n += (v >= 32767 || v <= -32768) ? 1u : 0u;
  }
};
// every lane of the warp calls it (lanes without rows contribute zeros)
F5_DEV void rstat_flush(unsigned long long *p, const RStat &s) {
  const unsigned mx = __reduce_max_sync(0xffffffffu, s.mx);
  const unsigned n = __reduce_add_sync(0xffffffffu, s.n);
  if ((threadIdx.x & 31) == 0) {
    if (mx) atomicMax(p, (unsigned long long)mx);
    if (n) atomicAdd(p + 1, (unsigned long long)n);
  }
}

// T_known >= 0: the step's token count, known to the caller (GM_CONV then
// skips reading *sg.T).  PERSIST: the persistent kernel's copy, without the
// GM_Y32 / GM_TO64 cases that its step program never emits (an unexpected
// mode raises DERR_RANGE): every line of code in that one-function kernel
// costs instruction-cache room between its phases.
template <bool PERSIST = false>
F5_DEV void epilogue_row(const GemvArgs &a, const GemvSeg &sg, int row, long long acc16, int e_x,
                         int in_f, unsigned long long &best, uint32_t epoch = 0, RStat *rs = nullptr,
                         int T_known = -1) {
  long long pex;
  const int32_t y = finish_y32(acc16, a.sh, a.err, &pex);
  const int orow = sg.out_row0 + row;
  if (sg.mode == GM_ARGMAX) {
    const unsigned long long k = argmax_key(y, orow);
    best = k > best ? k : best;
    if (sg.out) static_cast<int32_t *>(sg.out)[orow] = y;   // optional logits
    return;
  }
  if (sg.p_out) sg.p_out[orow] = pex;
  const int sh2 = (15 - sg.e - a.sh) - e_x + in_f - sg.out_f;
  const uint32_t tag = (epoch && sg.tag_op1) ? mk_tag(epoch, sg.tag_op1) : 0u;
  switch (sg.mode) {
    case GM_Y32:
      if constexpr (PERSIST) atomicOr(a.err, DERR_RANGE);
      else static_cast<int32_t *>(sg.out)[orow] = y;
      break;
    case GM_TO16: {
      const int32_t v = clip16(shift_to(y, sh2));
      if (tag) st_tagged(a, static_cast<uint32_t *>(sg.out) + orow, tag_word(tag, v));
      else static_cast<int16_t *>(sg.out)[orow] = (int16_t)v;
    } break;
    case GM_TO64:
      if constexpr (PERSIST) atomicOr(a.err, DERR_RANGE);
      else static_cast<int64_t *>(sg.out)[orow] = shift_to(y, sh2);
      break;
    case GM_RESID: {
      int32_t nv;
      if (tag) {   // the row's previous word was written by this CTA (same row partition)
        uint32_t *o = static_cast<uint32_t *>(sg.out) + orow;
        nv = clip16((int64_t)tag_s16(__ldcg(o)) + clip16(shift_to(y, sh2)));
        st_tagged(a, o, tag_word(tag, nv));
      } else {
        int16_t *o = static_cast<int16_t *>(sg.out) + orow;   // written by other CTAs: read at L2
        nv = clip16((int64_t)__ldcg(o) + clip16(shift_to(y, sh2)));
        *o = (int16_t)nv;
      }
      if (rs) rs->add(nv);
    } break;
    case GM_CONV: {   // ref/layer_fixed.py:1511-1520 for channel orow
      const long long v = clip16(shift_to(y, sh2));
      if (sg.out) static_cast<int16_t *>(sg.out)[orow] = (int16_t)v;
      int16_t *ring = static_cast<int16_t *>(sg.aux0) + (size_t)orow * 4;
      // cached loads: the ring word is touched only by this row's epilogue
      // (this step's write below, the next step's read in a later launch)
      const int4 cw = *reinterpret_cast<const int4 *>(static_cast<const int32_t *>(sg.aux1) + (size_t)orow * 4);
      const int T = T_known >= 0 ? T_known : *sg.T;
      const uint2 rw = *reinterpret_cast<const uint2 *>(ring);   // 4 int16 slots
      const int32_t qc = conv_silu(v, rw, cw, T);
      if (tag) st_tagged(a, static_cast<uint32_t *>(sg.aux_out) + orow, tag_word(tag, qc));
      else static_cast<int16_t *>(sg.aux_out)[orow] = (int16_t)qc;
      ring[T & 3] = (int16_t)v;
    } break;
    case GM_GATE_B: {   // ref/layer_fixed.py:1531; beta in [0, 2^15]: a tagged word holds it unsigned
      const long long v = clip16(shift_to(y, sh2));
      if (sg.out) static_cast<int16_t *>(sg.out)[orow] = (int16_t)v;
      const int32_t beta = (int32_t)sigmoid_q(v);
      if (tag) st_tagged(a, static_cast<uint32_t *>(sg.aux_out) + orow, tag_word(tag, beta));
      else static_cast<int32_t *>(sg.aux_out)[orow] = beta;
    } break;
    case GM_GATE_A: {   // ref/layer_fixed.py:1532-1538
      const long long v = clip16(shift_to(y, sh2));
      if (sg.out) static_cast<int16_t *>(sg.out)[orow] = (int16_t)v;
      const int32_t d = decay_gate(v, static_cast<const int32_t *>(sg.aux0)[orow],
                                   static_cast<const int32_t *>(sg.aux1)[orow]);
      if (tag) st_tagged(a, static_cast<uint32_t *>(sg.aux_out) + orow, tag_word(tag, d));
      else static_cast<int32_t *>(sg.aux_out)[orow] = d;
    } break;
    default: break;
  }
}

// MLP gate/up pair (ref/layer_fixed.py:1597-1602)
F5_DEV void epilogue_pair(const GemvArgs &a, const GemvSeg &sg, int row, long long accg, long long accu,
                          int e_x, int in_f, uint32_t epoch = 0) {
  const int32_t yg = finish_y32(accg, a.sh, a.err, nullptr);
  const int32_t yu = finish_y32(accu, a.sh, a.err, nullptr);
  const int64_t gq = shift_to(yg, (15 - sg.e - a.sh) - e_x + in_f - sg.out_f);
  const int64_t uq = shift_to(yu, (15 - sg.e2 - a.sh) - e_x + in_f - sg.out_f2);
  const int64_t sgv = clip16(silu_q(clip(gq, -(1 << 20), (1 << 20) - 1)));
  const int32_t v = clip16(rshr(sgv * uq, 12));
  if (epoch && sg.tag_op1) st_tagged(a, static_cast<uint32_t *>(sg.out) + sg.out_row0 + row, tag_word(mk_tag(epoch, sg.tag_op1), v));
  else static_cast<int16_t *>(sg.out)[sg.out_row0 + row] = (int16_t)v;
}

}  // namespace f5
