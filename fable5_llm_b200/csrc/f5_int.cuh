// Device integer primitives of the fixed-point decode law (sm_100a).
//
// Each function restates one reference function of coreyhahn/fable5_llm
// (cited file:line).  All arithmetic is two's-complement int64 with
// arithmetic (floor) right shifts, which is exactly Python's `>>` on ints and
// numpy's on int64; products are bounded well below 2^63 (bounds noted).
#pragma once
#include <stdint.h>
#include "f5_luts.h"

#define F5_DEV __device__ __forceinline__

// LUTs in global memory (read through L1): divergent per-lane indices make
// __constant__ serialise, so plain device arrays are used.
static __device__ const int32_t f5_lut_rsqrt[F5_LUT_RSQRT_N] = F5_LUT_RSQRT_INIT;
static __device__ const int32_t f5_lut_recip[F5_LUT_RECIP_N] = F5_LUT_RECIP_INIT;
static __device__ const int32_t f5_lut_exp2[F5_LUT_EXP2_N] = F5_LUT_EXP2_INIT;
static __device__ const int32_t f5_lut_sigmoid[F5_LUT_SIGMOID_N] = F5_LUT_SIGMOID_INIT;
static __device__ const int32_t f5_lut_softplus[F5_LUT_SOFTPLUS_N] = F5_LUT_SOFTPLUS_INIT;

// The arrays the lookups below read.  A translation unit whose kernels keep
// their own copy of the tables (the persistent decode kernel holds them in
// shared memory) defines these names before including this header.
#ifndef F5_LUT_RSQRT
#define F5_LUT_RSQRT f5_lut_rsqrt
#define F5_LUT_RECIP f5_lut_recip
#define F5_LUT_EXP2 f5_lut_exp2
#define F5_LUT_SIGMOID f5_lut_sigmoid
#define F5_LUT_SOFTPLUS f5_lut_softplus
#endif

namespace f5 {

// fixed-point formats of the 9B operating point (ref/layer_fixed.py:103-147,404)
constexpr int RS_F = 7, QKV_F = 8, NRM_F = 14, S_F = 13, GAT_F = 15, CW_F = 13,
              ROPE_F = 15, DN_NORM_F = 11;
constexpr int M_Q15_MAX = 65535;
constexpr int64_t EPS_M = 1099512;   // round(1e-6 * 2^40), ref/layer_fixed.py:650
constexpr int EPS_Q = 40;

// ref/w4a8_ref.py:90-99 rshift_round: round half away from zero; s<0 = exact <<.
// For s > 0 it is computed branch-free as floor((v + 2^(s-1) - [v < 0]) / 2^s)
// (an arithmetic shift): for v < 0, -floor((-v + 2^(s-1)) / 2^s) =
// floor((v - 2^(s-1)) / 2^s + 1 - 2^-s) = floor((v + 2^(s-1) - 1) / 2^s).
F5_DEV int64_t rshr(int64_t v, int s) {
  if (s <= 0) return s == 0 ? v : (int64_t)((uint64_t)v << (-s));
  return (v + ((int64_t)1 << (s - 1)) - (int64_t)(v < 0)) >> s;
}
// 32-bit form for operands known to fit (|v| + 2^(s-1) < 2^31), 0 < s < 31.
F5_DEV int32_t rshr32p(int32_t v, int s) {
  return (v + (1 << (s - 1)) - (int32_t)(v < 0)) >> s;
}
F5_DEV int64_t clip(int64_t v, int64_t lo, int64_t hi) { return v < lo ? lo : (v > hi ? hi : v); }
F5_DEV int32_t clip16(int64_t v) { return (int32_t)clip(v, -32768, 32767); }  // ref/layer_fixed.py:809
F5_DEV int bitlen(uint64_t v) { return v ? 64 - __clzll((long long)v) : 0; }
F5_DEV uint64_t uabs(int64_t v) { return v < 0 ? (uint64_t)(-v) : (uint64_t)v; }

// ref/fixedpoint.py:24-33 dyn_quant_i8: smallest e with (m + (1<<e>>1)) >> e <= 127
// the smallest e with (m + (1 << e >> 1)) >> e <= 127: for m > 127 it is
// e0 = bitlen(m) - 7 (m >> e0 in [64, 127]) or e0 + 1 when the rounding
// carries past 127; e0 - 1 never suffices (m >> (e0 - 1) >= 128)
F5_DEV int dynq8_e(uint64_t m) {
  if (m <= 127ull) return 0;
  const int e0 = 64 - __clzll((long long)m) - 7;
  return e0 + (((m + (1ull << (e0 - 1))) >> e0) > 127ull ? 1 : 0);
}
F5_DEV int32_t dynq8_apply(int64_t x, int e) { return (int32_t)clip(e ? rshr(x, e) : x, -127, 127); }
// dynq8_apply for |x| < 2^30 in 32-bit arithmetic: sign(x) * min((|x| +
// 2^(e-1)) >> e, 127) is round-half-away-from-zero then clip to +-127.
F5_DEV int32_t dynq8_apply32(int32_t x, int e) {
  const int32_t ax = x < 0 ? -x : x;
  int32_t r = (ax + ((1 << e) >> 1)) >> e;
  r = r < 127 ? r : 127;
  return x < 0 ? -r : r;
}

// Pull the LUTs' cache lines into L1 (thread t in [0, 51) takes one line):
// issued at the start of a phase that will look them up, so the lookups on
// its dependency chain hit L1 even after an acquire invalidated it.
F5_DEV void lut_prefetch_l1(int t) {
  const char *p = nullptr;
  if (t < 16) p = reinterpret_cast<const char *>(f5_lut_rsqrt) + t * 128;
  else if (t < 24) p = reinterpret_cast<const char *>(f5_lut_recip) + (t - 16) * 128;
  else if (t < 33) p = reinterpret_cast<const char *>(f5_lut_exp2) + (t - 24) * 128;
  else if (t < 42) p = reinterpret_cast<const char *>(f5_lut_sigmoid) + (t - 33) * 128;
  else if (t < 51) p = reinterpret_cast<const char *>(f5_lut_softplus) + (t - 42) * 128;
  if (p) asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// ref/layer_fixed.py:442-467 bf_shift (guard 0)
F5_DEV int bf_shift(uint64_t m) {
  if (m == 0) return 0;
  int k = bitlen(m) - 15;
  if (k > 0 && rshr((int64_t)m, k) > 32767) ++k;
  return k;
}

// ref/fixedpoint.py:56-75 rsqrt_q.  v > 0 (< 2^62).  m < 2^32, r <= ~2^30:
// r*r < 2^61, m*r2 < 2^62, r*(3<<30 - mr2) < 2^62.
F5_DEV void rsqrt_q(uint64_t v, int P, int64_t &r_out, int &e_out) {
  int s = bitlen(v) - 32;
  if (((s - P) & 1) != 0) s += 1;
  const uint64_t m = s >= 0 ? (v >> s) : (v << (-s));
  const int E = s - P + 30;
  const int idx = m < (1ull << 31) ? (int)((m >> 22) & 0xFF) : (256 | (int)((m >> 23) & 0xFF));
  int64_t r = (int64_t)F5_LUT_RSQRT[idx] << 15;
  const int64_t mi = (int64_t)m;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int64_t r2 = (r * r) >> 30;
    const int64_t mr2 = (mi * r2) >> 30;
    r = (r * ((3ll << 30) - mr2)) >> 31;
  }
  r_out = r;
  e_out = -(E / 2);   // E is even: exact, equal to Python's -E // 2
}

// ref/fixedpoint.py:179-198 recip_q.  v > 0.  m < 2^31, r <= 2^30.
F5_DEV void recip_q(uint64_t v, int P, int64_t &r_out, int &e_out) {
  const int n = bitlen(v);
  const int sh = n - 31;
  const uint64_t m = sh >= 0 ? (v >> sh) : (v << (-sh));
  int64_t idx = ((int64_t)m - (1ll << 30)) >> 22;
  if (idx > 255) idx = 255;
  int64_t r = (int64_t)F5_LUT_RECIP[idx] << 15;
  const int64_t mi = (int64_t)m;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int64_t mr = (mi * r) >> 30;
    r = (r * ((2ll << 30) - mr)) >> 30;
  }
  r_out = r;
  e_out = -(sh + 30 - P);
}

// ref/fixedpoint.py:99-106 exp2_frac_q16, f in [0, 2^16)
// (table entries < 2^18, lo < 2^8: the interpolation fits 32-bit integers)
F5_DEV int64_t exp2_frac_q16(int64_t f) {
  const int i = (int)(f >> 8), lo = (int)(f & 0xFF);
  const int32_t a = F5_LUT_EXP2[i], b = F5_LUT_EXP2[i + 1];
  return (int64_t)(a + (((b - a) * lo + 128) >> 8));
}

// ref/fixedpoint.py:109-121 exp_neg_q: x <= 0 in Q16 -> Q30.  |x| < 2^45.
F5_DEV int64_t exp_neg_q(int64_t x) {
  const int64_t t = (x * 94548) >> 16;
  const int64_t n = (-t + 0xFFFF) >> 16;
  const int64_t f = t + (n << 16);
  if (n >= 31) return 0;
  const int64_t v = exp2_frac_q16(f);
  return n <= 14 ? (v << (14 - n)) : (v >> (n - 14));
}

// ref/fixedpoint.py:135-147 sigmoid_q: Q12 -> Q15, PWL over [-16, 16)
// (entries <= 32767, lo < 2^9: the interpolation fits 32-bit integers)
F5_DEV int64_t sigmoid_q(int64_t x) {
  const int32_t xc = (int32_t)clip(x, -(16 << 12), (16 << 12) - 1);
  const int u = xc + (16 << 12);
  const int i = u >> 9, lo = u & 0x1FF;
  const int32_t a = F5_LUT_SIGMOID[i], b = F5_LUT_SIGMOID[i + 1];
  return (int64_t)(a + (((b - a) * lo + 256) >> 9));
}

// ref/fixedpoint.py:150-165 softplus_q: Q12 -> Q12
F5_DEV int64_t softplus_q(int64_t x) {
  if (x >= (16 << 12)) return x;
  if (x < -(16 << 12)) return 0;
  const int u = (int)(x + (16 << 12));
  const int i = u >> 9, lo = u & 0x1FF;
  const int32_t a = F5_LUT_SOFTPLUS[i], b = F5_LUT_SOFTPLUS[i + 1];   // < 2^17: 32-bit interpolation
  return (int64_t)(a + (((b - a) * lo + 256) >> 9));
}

// ref/fixedpoint.py:168-171 silu_q = rshr(x * sigmoid_q(x), 15)
// x * sigmoid_q(x) as one 32 x 32 -> 64-bit multiply whenever x fits int32
// (always on the decode path: |x| <= 2^21)
F5_DEV int64_t silu_q(int64_t x) {
  const int64_t sg = sigmoid_q(x);
  const int64_t p = (x == (int64_t)(int32_t)x) ? (int64_t)(int32_t)x * (int32_t)sg : x * sg;
  return rshr(p, 15);
}

// ref/layer_fixed.py:1224-1236 second shift of matvec_to, either direction
F5_DEV int64_t shift_to(int64_t y32, int sh2) { return sh2 >= 0 ? rshr(y32, sh2) : (int64_t)((uint64_t)y32 << (-sh2)); }

// ref/layer_fixed.py:509-546 dn_norm_scale: float64 host scale, IEEE
// correctly-rounded ops (explicit _rn intrinsics: no contraction), Python
// round() = half-to-even (__double2ll_rn).  ss is the numpy int64 (wrapping)
// sum; int64 -> double is round-to-nearest-even like Python's float(int).
F5_DEV int32_t dn_norm_scale(int64_t ss, int k_h, int n) {
  const double ssd = __ll2double_rn(ss);
  const double mean = __ddiv_rn(__ddiv_rn(ssd, 67108864.0 /* 2^(2*S_F) */), (double)n);
  const double s = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(mean, 1e-6)));
  const double A = __dmul_rn(s, 0.25);                 // 2^(DN_NORM_F - S_F)
  // 2^(15+k_h) built from its exponent bits (k_h in [-14, 17]): exact scale
  const double p2 = __longlong_as_double((long long)(1023 + 15 + k_h) << 52);
  const long long m = __double2ll_rn(__dmul_rn(A, p2));  // half-to-even
  return (int32_t)clip(m, 0, M_Q15_MAX);
}

// ref/layer_fixed.py:681-691 eps_ss_addend (in_f = S_F, n_log2 = 7)
F5_DEV int64_t eps_ss_addend(int k, int in_f, int n_log2) {
  return rshr(EPS_M, EPS_Q - (2 * (in_f - k) + n_log2));
}

// ref/layer_fixed.py:694-767 eps_norm_scale over an int16 block (ss given)
F5_DEV int32_t eps_norm_scale(int64_t ss16, int k, int n_log2) {
  int64_t v = ss16 + eps_ss_addend(k, S_F, n_log2);
  if (v <= 0) v = 1;
  int64_t r; int e;
  rsqrt_q((uint64_t)v, 2 * S_F + n_log2, r, e);
  const int sh = S_F - DN_NORM_F + 15 - e;
  return (int32_t)clip(rshr(r, sh), 0, M_Q15_MAX);
}

}  // namespace f5
