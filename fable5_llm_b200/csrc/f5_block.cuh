// Block-level integer reductions shared by the vector kernels.
#pragma once
#include "f5_int.cuh"

namespace f5 {

// Sum over the block (any blockDim multiple of 32, <= 1024).  `red` holds
// >= 32 long longs of shared scratch.  Result valid in every thread.
F5_DEV long long block_sum_ll(long long v, long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  long long t = 0;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

F5_DEV unsigned long long block_sum_ull(unsigned long long v, unsigned long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  unsigned long long t = 0;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

F5_DEV unsigned long long block_max_ull(unsigned long long v, unsigned long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  unsigned long long t = 0;
  for (int i = 0; i < nw; ++i) t = red[i] > t ? red[i] : t;
  return t;
}

F5_DEV long long block_max_ll(long long v, long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  long long t = red[0];
  for (int i = 1; i < nw; ++i) t = red[i] > t ? red[i] : t;
  return t;
}

// ---- sync policies: the same reduction code over the whole block
// (__syncthreads) or over a thread group with a named barrier ----
struct BlockSync {
  F5_DEV int tid() const { return threadIdx.x; }
  F5_DEV int n() const { return blockDim.x; }
  F5_DEV void sync() const { __syncthreads(); }
  F5_DEV bool any(bool p) const { return __syncthreads_or(p) != 0; }
};
// group = threads [BASE, BASE+N) of the block, barrier id ID (N % 32 == 0)
template <int ID, int N, int BASE = 0>
struct NamedSync {
  F5_DEV int tid() const { return (int)threadIdx.x - BASE; }
  F5_DEV int n() const { return N; }
  F5_DEV void sync() const { asm volatile("bar.sync %0, %1;" ::"n"(ID), "n"(N) : "memory"); }
  // group-uniform OR of a predicate (also a barrier)
  F5_DEV bool any(bool p) const {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n bar.red.or.pred po, %2, %3, pi;\n"
        " selp.u32 %0, 1, 0, po;\n}"
        : "=r"(r) : "r"((uint32_t)p), "n"(ID), "n"(N) : "memory");
    return r != 0;
  }
};

// Sum over the group of per-thread values |v| < 2^40 with two 32-bit
// redux.sync adds per warp (v = hi * 2^22 + lo, lo in [0, 2^22)): exact.
// The cross-warp stage of every group reduction below is parallel: after
// the partials are published, each warp reads them one per lane (lanes
// beyond the warp count read the identity) and reduces them itself, instead
// of a serial loop over the partials on every thread's dependency chain.
F5_DEV long long warp_sum_s64(long long v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <class SY>
F5_DEV long long g_sum_split(const SY &sy, long long v, long long *red) {
  const unsigned slo = __reduce_add_sync(0xffffffffu, (unsigned)v & 0x3FFFFFu);
  const int shi = __reduce_add_sync(0xffffffffu, (int)(v >> 22));
  const long long w = ((long long)shi << 22) + (long long)slo;
  const int wi = sy.tid() >> 5, nw = sy.n() >> 5, lane = sy.tid() & 31;
  sy.sync();
  if (lane == 0) red[wi] = w;
  sy.sync();
  // warp partials are < 2^45 in magnitude (32 lanes of < 2^40): split again
  const long long p = lane < nw ? red[lane] : 0;
  const unsigned plo = __reduce_add_sync(0xffffffffu, (unsigned)p & 0x3FFFFFu);
  const long long phi = warp_sum_s64(p >> 22);
  return (phi << 22) + (long long)plo;
}
// Two sums (|a|, |b| < 2^40 per thread) in one barrier round.
template <class SY>
F5_DEV void g_sum2_split(const SY &sy, long long a, long long b, long long *red, long long &sa, long long &sb) {
  const long long wa = ((long long)__reduce_add_sync(0xffffffffu, (int)(a >> 22)) << 22) +
                       (long long)__reduce_add_sync(0xffffffffu, (unsigned)a & 0x3FFFFFu);
  const long long wb = ((long long)__reduce_add_sync(0xffffffffu, (int)(b >> 22)) << 22) +
                       (long long)__reduce_add_sync(0xffffffffu, (unsigned)b & 0x3FFFFFu);
  const int wi = sy.tid() >> 5, nw = sy.n() >> 5, lane = sy.tid() & 31;
  sy.sync();
  if (lane == 0) {
    red[wi] = wa;
    red[32 + wi] = wb;
  }
  sy.sync();
  const long long pa = lane < nw ? red[lane] : 0, pb = lane < nw ? red[32 + lane] : 0;
  sa = ((warp_sum_s64(pa >> 22)) << 22) + (long long)__reduce_add_sync(0xffffffffu, (unsigned)pa & 0x3FFFFFu);
  sb = ((warp_sum_s64(pb >> 22)) << 22) + (long long)__reduce_add_sync(0xffffffffu, (unsigned)pb & 0x3FFFFFu);
}
// Max of u64 a and wrapping u64 sum of b in one barrier round.
template <class SY>
F5_DEV void g_max_sum_ull(const SY &sy, unsigned long long a, unsigned long long b, unsigned long long *red,
                          unsigned long long &ma, unsigned long long &sb) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, a, o);
    a = t > a ? t : a;
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int wi = sy.tid() >> 5, nw = sy.n() >> 5, lane = sy.tid() & 31;
  sy.sync();
  if (lane == 0) {
    red[wi] = a;
    red[32 + wi] = b;
  }
  sy.sync();
  a = lane < nw ? red[lane] : 0ull;
  b = lane < nw ? red[32 + lane] : 0ull;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, a, o);
    a = t > a ? t : a;
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  ma = a;
  sb = b;
}

// Two u64 maxima in one barrier round.
template <class SY>
F5_DEV void g_max2_ull(const SY &sy, unsigned long long a, unsigned long long b, unsigned long long *red,
                       unsigned long long &ma, unsigned long long &mb) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, a, o), u = __shfl_xor_sync(0xffffffffu, b, o);
    a = t > a ? t : a;
    b = u > b ? u : b;
  }
  const int wi = sy.tid() >> 5, nw = sy.n() >> 5, lane = sy.tid() & 31;
  sy.sync();
  if (lane == 0) {
    red[wi] = a;
    red[32 + wi] = b;
  }
  sy.sync();
  a = lane < nw ? red[lane] : 0ull;
  b = lane < nw ? red[32 + lane] : 0ull;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, a, o), u = __shfl_xor_sync(0xffffffffu, b, o);
    a = t > a ? t : a;
    b = u > b ? u : b;
  }
  ma = a;
  mb = b;
}

// Max over the group of 32-bit unsigned values (redux.sync.max per warp).
template <class SY>
F5_DEV unsigned g_max_u32(const SY &sy, unsigned v, long long *red) {
  v = __reduce_max_sync(0xffffffffu, v);
  const int wi = sy.tid() >> 5, nw = sy.n() >> 5, lane = sy.tid() & 31;
  sy.sync();
  if (lane == 0) red[wi] = v;
  sy.sync();
  return __reduce_max_sync(0xffffffffu, lane < nw ? (unsigned)red[lane] : 0u);
}

template <class SY>
F5_DEV long long g_sum_ll(const SY &sy, long long v, long long *red) {
  v = warp_sum_s64(v);
  const int w = sy.tid() >> 5, nw = sy.n() >> 5, lane = sy.tid() & 31;
  sy.sync();
  if (lane == 0) red[w] = v;
  sy.sync();
  return warp_sum_s64(lane < nw ? red[lane] : 0);
}
template <class SY>
F5_DEV unsigned long long g_sum_ull(const SY &sy, unsigned long long v, unsigned long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = sy.tid() >> 5, nw = sy.n() >> 5, lane = sy.tid() & 31;
  sy.sync();
  if (lane == 0) red[w] = v;
  sy.sync();
  unsigned long long t = lane < nw ? red[lane] : 0ull;   // wrapping sums: order-free modulo 2^64
#pragma unroll
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}
template <class SY>
F5_DEV unsigned long long g_max_ull(const SY &sy, unsigned long long v, unsigned long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  const int w = sy.tid() >> 5, nw = sy.n() >> 5, lane = sy.tid() & 31;
  sy.sync();
  if (lane == 0) red[w] = v;
  sy.sync();
  unsigned long long t = lane < nw ? red[lane] : 0ull;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long u = __shfl_xor_sync(0xffffffffu, t, o);
    t = u > t ? u : t;
  }
  return t;
}

// Reduce four per-lane values over the warp with six shuffles instead of
// twenty: afterwards every lane of the 8-lane group g = lane >> 3 holds the
// warp total of v[g].  Integer sums are order-free, so the result equals
// four separate butterflies.
F5_DEV int warp_sum4_i32(const int (&v)[4]) {
  const int lane = threadIdx.x & 31;
  const bool b4 = lane & 16, b3 = lane & 8;
  int k0 = b4 ? v[2] : v[0], k1 = b4 ? v[3] : v[1];
  k0 += __shfl_xor_sync(0xffffffffu, b4 ? v[0] : v[2], 16);
  k1 += __shfl_xor_sync(0xffffffffu, b4 ? v[1] : v[3], 16);
  int k = b3 ? k1 : k0;
  k += __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
  k += __shfl_xor_sync(0xffffffffu, k, 4);
  k += __shfl_xor_sync(0xffffffffu, k, 2);
  k += __shfl_xor_sync(0xffffffffu, k, 1);
  return k;
}

}  // namespace f5
