// Batch-1 W4A8 GEMV over the reference's packed DDR row format (sm_100a).
//
// Law (ref/w4a8_ref.py:254-289 matvec_y32):
//   acc_g = sum_{k in group g} w4[k] * x8[k]      (int32)
//   p     = sum_g m_g * acc_g                      (int64, < 2^41)
//   y32   = rshift_round(p, sh)
// followed by a fused epilogue (ref/layer_fixed.py:1224-1236 matvec_to's
// second shift, clip16, residual add, the MLP silu*up product of
// ref/layer_fixed.py:1597-1604, or the LM-head running argmax of
// ref/gen_model_script.py:641).
//
// Memory layout: the weights stay in the reference's own row format
// (ref/w4a8_ref.py:102-114: K/128 64-byte weight beats, low nibble = even k,
// then ceil(NG/32) beats of little-endian uint16 group mantissas), i.e.
// exactly 4.125 bits/weight, 64-byte aligned rows.  A row is streamed by one
// warp with 16-byte non-allocating loads: lane l of chunk c reads bytes
// [c*512 + 16l, +16) = weights k in [c*1024 + 32l, +32).  A 16-byte load
// never straddles a group (g = 128 or 64).
//
// Nibble arithmetic: (word << 4) & 0xF0F0F0F0 puts each even-k nibble in the
// high half of its byte, which read as int8 is 16*w; word & 0xF0F0F0F0 does
// the same for odd k.  Two dp4a against the even/odd-permuted x8 bytes give
// 16*sum(w*x) exactly; the factor 16 is removed once per row (p16 >> 4 is
// exact because every term is a multiple of 16).  The int64 group-scale FMA
// m_g * acc is applied per lane-chunk (linear, so summing partial group sums
// times m_g equals m_g times the group sum -- integer arithmetic is exact
// and order-free).
#include "f5_block.cuh"
#include "f5_kernels.cuh"
#include "f5_tma.cuh"

namespace f5 {

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
    const longlong2 u = *reinterpret_cast<const longlong2 *>(p + j);
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

// rmsnorm_fx element (ref/layer_fixed.py:1242-1278): clip33(rshr(x*r, 30-e)) * gain
F5_DEV long long rms_elem(long long x, long long r, int e, long long gain) {
  long long y = rshr(x * r, 30 - e);
  y = clip(y, -(1ll << 32), (1ll << 32) - 1);
  return clip16(rshr(y * gain, 14));
}

// element j (0..7) of 8 int16 packed in a uint4
F5_DEV long long get16(const uint4 &u, int j) {
  const uint32_t w = (j >> 1) == 0 ? u.x : ((j >> 1) == 1 ? u.y : ((j >> 1) == 2 ? u.z : u.w));
  return (long long)(int16_t)((j & 1) ? (w >> 16) : (w & 0xFFFFu));
}

// Redundant per-CTA computation of the GEMV's quantized input (see GemvPro).
// Every value is read from global memory once and held in registers across
// the reduction passes (MAXB 8-element blocks per thread).
template <int MAXB>
F5_DEV void prologue(const GemvArgs &a, uint2 *xs, long long *red, long long *s_r, int *s_meta) {
  const int tid = threadIdx.x, BT = blockDim.x, K = a.K, nblk = K >> 3;
  const GemvPrologue &P = a.pro;
  const bool store = (P.xq_out.x8 != nullptr) && blockIdx.x == 0;
  long long q[8];
  if (P.mode == PRO_RMSNORM || P.mode == PRO_DYNQ8) {
    const int16_t *src = static_cast<const int16_t *>(P.src);
    uint4 raw[MAXB];
#pragma unroll
    for (int j = 0; j < MAXB; ++j) {
      const int b = tid + j * BT;
      raw[j] = b < nblk ? *reinterpret_cast<const uint4 *>(src + 8 * b) : make_uint4(0, 0, 0, 0);
    }
    if constexpr (MAXB <= 2) {
      if (P.mode == PRO_RMSNORM) {     // ref/layer_fixed.py:1242-1278 (H = 4096)
        int4 wl[MAXB][2];
#pragma unroll
        for (int j = 0; j < MAXB; ++j) {
          const int b = tid + j * BT;
          wl[j][0] = b < nblk ? *reinterpret_cast<const int4 *>(P.w + 8 * b) : make_int4(0, 0, 0, 0);
          wl[j][1] = b < nblk ? *reinterpret_cast<const int4 *>(P.w + 8 * b + 4) : make_int4(0, 0, 0, 0);
        }
        long long ss = 0;
#pragma unroll
        for (int j = 0; j < MAXB; ++j)
#pragma unroll
          for (int k = 0; k < 8; ++k) { const long long v = get16(raw[j], k); ss += v * v; }
        ss = block_sum_ll(ss, red);
        if (tid == 0) {
          int64_t r; int e;
          rsqrt_q((uint64_t)(ss == 0 ? 1 : ss), 2 * P.in_f + (31 - __clz(K)), r, e);
          *s_r = r;
          s_meta[2] = e;
        }
        __syncthreads();
        const long long r = *s_r;
        const int e = s_meta[2];
        const long long add1 = P.one_plus ? (1 << 14) : 0;
#pragma unroll
        for (int j = 0; j < MAXB; ++j) {
          const int wv[8] = {wl[j][0].x, wl[j][0].y, wl[j][0].z, wl[j][0].w,
                             wl[j][1].x, wl[j][1].y, wl[j][1].z, wl[j][1].w};
          uint32_t pk[4];
#pragma unroll
          for (int k = 0; k < 8; k += 2) {
            const long long x0 = rms_elem(get16(raw[j], k), r, e, wv[k] + add1);
            const long long x1 = rms_elem(get16(raw[j], k + 1), r, e, wv[k + 1] + add1);
            pk[k >> 1] = ((uint32_t)x0 & 0xFFFFu) | ((uint32_t)x1 << 16);
          }
          raw[j] = make_uint4(pk[0], pk[1], pk[2], pk[3]);   // normalised, int16
        }
      }
    } else {
      if (P.mode == PRO_RMSNORM && tid == 0) atomicOr(a.err, DERR_RANGE);   // RMSNorm is bound to K <= 4096
    }
    unsigned long long mx = 0;
#pragma unroll
    for (int j = 0; j < MAXB; ++j)
#pragma unroll
      for (int k = 0; k < 8; ++k) { const unsigned long long m = uabs(get16(raw[j], k)); mx = m > mx ? m : mx; }
    mx = block_max_ull(mx, reinterpret_cast<unsigned long long *>(red));
    const int ex = dynq8_e(mx);
#pragma unroll
    for (int j = 0; j < MAXB; ++j) {
      const int b = tid + j * BT;
      if (b < nblk) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          q[k] = dynq8_apply(get16(raw[j], k), ex);
          if (store) P.xq_out.x8[8 * b + k] = (int8_t)q[k];
        }
        put8(xs, b, q);
      }
    }
    if (tid == 0) { s_meta[0] = ex; s_meta[1] = P.in_f; }
  } else if constexpr (MAXB <= 2) {  // PRO_ATTN_GATE (ref/layer_fixed.py:1441-1449); K = NQ*HD = 4096
    const int64_t *src = static_cast<const int64_t *>(P.src);
    long long v[MAXB][8];
#pragma unroll
    for (int j = 0; j < MAXB; ++j) {
      const int b = tid + j * BT;
      if (b < nblk) load8_i64(src + 8 * b, v[j]);
      else
#pragma unroll
        for (int k = 0; k < 8; ++k) v[j][k] = 0;
    }
    unsigned long long mx = 0;
#pragma unroll
    for (int j = 0; j < MAXB; ++j)
#pragma unroll
      for (int k = 0; k < 8; ++k) { const unsigned long long m = uabs(v[j][k]); mx = m > mx ? m : mx; }
    mx = block_max_ull(mx, reinterpret_cast<unsigned long long *>(red));
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
    mg = block_max_ull(mg, reinterpret_cast<unsigned long long *>(red));
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
F5_DEV void epilogue_row(const GemvArgs &a, const GemvSeg &sg, int row, long long acc16, int e_x,
                         int in_f, unsigned long long &best) {
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
  switch (sg.mode) {
    case GM_Y32: static_cast<int32_t *>(sg.out)[orow] = y; break;
    case GM_TO16: static_cast<int16_t *>(sg.out)[orow] = (int16_t)clip16(shift_to(y, sh2)); break;
    case GM_TO64: static_cast<int64_t *>(sg.out)[orow] = shift_to(y, sh2); break;
    case GM_RESID: {
      int16_t *o = static_cast<int16_t *>(sg.out) + orow;
      *o = (int16_t)clip16((int64_t)*o + clip16(shift_to(y, sh2)));
    } break;
    default: break;
  }
}

// MLP gate/up pair (ref/layer_fixed.py:1597-1602)
F5_DEV void epilogue_pair(const GemvArgs &a, const GemvSeg &sg, int row, long long accg, long long accu,
                          int e_x, int in_f) {
  const int32_t yg = finish_y32(accg, a.sh, a.err, nullptr);
  const int32_t yu = finish_y32(accu, a.sh, a.err, nullptr);
  const int64_t gq = shift_to(yg, (15 - sg.e - a.sh) - e_x + in_f - sg.out_f);
  const int64_t uq = shift_to(yu, (15 - sg.e2 - a.sh) - e_x + in_f - sg.out_f2);
  const int64_t sgv = clip16(silu_q(clip(gq, -(1 << 20), (1 << 20) - 1)));
  static_cast<int16_t *>(sg.out)[sg.out_row0 + row] = (int16_t)clip16(rshr(sgv * uq, 12));
}

constexpr int GT_CONS = 16;                     // consumer warps
constexpr int GT_CTHREADS = GT_CONS * 32;
constexpr int GT_THREADS = GT_CTHREADS + 32;    // + one producer warp
constexpr int GT_MAX_STAGES = 4;
constexpr int GT_CTA_SMEM = 232448 - 6144;      // dynamic smem per CTA (one CTA per SM)
constexpr int GT_RES_MAX = 2048;                // deferred row results per CTA
constexpr unsigned long long GT_WAIT_NS = 2000000000ull;   // 2 s: a safety net only

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

// Persistent TMA-pipelined GEMV: a producer warp streams contiguous blocks
// of packed rows (cp.async.bulk, 16-byte aligned, no multicast) into
// shared-memory stages guarded by full/empty mbarriers; sixteen consumer
// warps reduce one row per warp out of shared memory, park the row's p16 in
// shared memory and release the stage at once.  The per-row epilogues run
// after the CTA's last chunk with every consumer thread taking one row, so
// the serial int64 epilogue never sits on the weight-stream critical path.
// The first stages are issued BEFORE griddepcontrol.wait: the weights do not
// depend on the previous kernel, so under programmatic dependent launch the
// weight stream overlaps the producer kernel's tail.
template <int NCH>
__global__ void __launch_bounds__(GT_THREADS, 1) k_gemv(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar_full[GT_MAX_STAGES], bar_empty[GT_MAX_STAGES];
  __shared__ long long red[32];
  __shared__ long long s_r;
  __shared__ int s_meta[4];
  __shared__ volatile int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K2 = a.K >> 1;
  const int gshift = (a.g == 128) ? 6 : 5;
  const int NS = a.stages;
  const uint32_t stage_bytes = (uint32_t)a.rows_per_stage * (uint32_t)a.stride;
  uint2 *xs = reinterpret_cast<uint2 *>(smem + NS * stage_bytes);
  long long *s_res = reinterpret_cast<long long *>(smem + NS * stage_bytes + NCH * 4 * 32 * sizeof(uint2));
  const int G = gridDim.x, b = blockIdx.x;
  const int u0 = (int)((long long)a.total_units * b / G);
  const int u1 = (int)((long long)a.total_units * (b + 1) / G);

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_empty[i], GT_CONS);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // producer: the first NS chunks need no empty-wait -> issue them now
  int pu = u0, pi = 0;
  if (warp == GT_CONS && lane == 0) {
    Chunk ch;
    while (pi < NS && next_chunk(a, pu, u1, ch)) {
      const GemvSeg &sg = a.seg[ch.seg];
      const uint32_t nb = (uint32_t)ch.n * a.stride;
      uint8_t *dst = smem + pi * stage_bytes;
      const bool pair = sg.mode == GM_SILU_MUL;
      mbar_expect_tx(&bar_full[pi], pair ? 2 * nb : nb);
      bulk_g2s(dst, sg.w + (size_t)ch.r0 * a.stride, nb, &bar_full[pi]);
      if (pair) bulk_g2s(dst + nb, sg.w2 + (size_t)ch.r0 * a.stride, nb, &bar_full[pi]);
      ++pi;
    }
  }

  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- prologue (all warps): x8 into the lane-major even/odd layout ----
  const int nblk = a.K >> 3;
  if (a.pro.mode == PRO_X8) {
    for (int bb = tid; bb < nblk; bb += blockDim.x) {
      const uint2 v = *reinterpret_cast<const uint2 *>(a.x8 + 8 * bb);
      uint2 o;
      o.x = __byte_perm(v.x, v.y, 0x6420);
      o.y = __byte_perm(v.x, v.y, 0x7531);
      xs[(((bb >> 7) << 2) + (bb & 3)) * 32 + ((bb >> 2) & 31)] = o;
    }
    if (tid == 0) {
      s_meta[0] = a.xmeta ? a.xmeta[0] : 0;
      s_meta[1] = a.xmeta ? a.xmeta[1] : 0;
    }
  } else {
    prologue<(NCH * 128 + GT_THREADS - 1) / GT_THREADS>(a, xs, red, &s_r, s_meta);
  }
  __syncthreads();
  const int e_x = s_meta[0], in_f = s_meta[1];

  if (warp == GT_CONS) {
    // ---- producer: remaining chunks, each after its stage is released ----
    if (lane == 0) {
      Chunk ch;
      int issued = pi;
      while (!s_abort && next_chunk(a, pu, u1, ch)) {
        const int s = issued % NS;
        if (!mbar_wait(&bar_empty[s], ((issued / NS) - 1) & 1, GT_WAIT_NS)) {
          s_abort = 1;
          atomicOr(a.err, DERR_TIMEOUT);
          break;
        }
        const GemvSeg &sg = a.seg[ch.seg];
        const uint32_t nb = (uint32_t)ch.n * a.stride;
        uint8_t *dst = smem + s * stage_bytes;
        const bool pair = sg.mode == GM_SILU_MUL;
        mbar_expect_tx(&bar_full[s], pair ? 2 * nb : nb);
        bulk_g2s(dst, sg.w + (size_t)ch.r0 * a.stride, nb, &bar_full[s]);
        if (pair) bulk_g2s(dst + nb, sg.w2 + (size_t)ch.r0 * a.stride, nb, &bar_full[s]);
        ++issued;
      }
      // never leave the CTA with copies in flight: drain every issued stage
      // the consumers have not waited on (bounded)
      if (s_abort) {
        for (int i = max(0, issued - NS); i < issued; ++i)
          mbar_wait(&bar_full[i % NS], (i / NS) & 1, GT_WAIT_NS);
      }
    }
    return;
  }

  // ---- consumers: one row per warp, results parked in s_res ----
  uint2 xr[4][4];
  if (NCH <= 4) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) xr[c][j] = c < NCH ? xs[((c << 2) + j) * 32 + lane] : make_uint2(0, 0);
  }
  int cu = u0, ci = 0;
  Chunk ch;
  while (next_chunk(a, cu, u1, ch)) {
    const int s = ci % NS;
    if (s_abort || !mbar_wait(&bar_full[s], (ci / NS) & 1, GT_WAIT_NS)) {
      if (!s_abort) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); }
      break;
    }
    const uint8_t *st = smem + s * stage_bytes;
    const bool pair = a.seg[ch.seg].mode == GM_SILU_MUL;
    const int nrows = pair ? 2 * ch.n : ch.n;
    const int cbase = ch.u - u0;
    for (int r = warp; r < nrows; r += GT_CONS) {
      const long long aa = warp_sum_ll(row_dot<NCH>(st + (size_t)r * a.stride, K2, gshift, lane, xr, xs));
      if (lane == 0) s_res[pair ? (r < ch.n ? 2 * (cbase + r) : 2 * (cbase + r - ch.n) + 1) : cbase + r] = aa;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar_empty[s]);
    ++ci;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(GT_CTHREADS) : "memory");
  if (s_abort) return;

  // ---- deferred epilogues: one unit per consumer thread ----
  unsigned long long best = 0ull;
  for (int i = tid; i < u1 - u0; i += GT_CTHREADS) {
    const int u = u0 + i;
    const GemvSeg &sg = a.seg[seg_of(a, u)];
    const int row = u - sg.unit_begin;
    if (sg.mode == GM_SILU_MUL) {
      epilogue_pair(a, sg, row, s_res[2 * i], s_res[2 * i + 1], e_x, in_f);
    } else {
      epilogue_row(a, sg, row, s_res[i], e_x, in_f, best);
    }
  }
  if (a.argmax_key) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    if (lane == 0 && best) atomicMax(a.argmax_key, best);
  }
}

int gemv_rows_per_stage(int stride) {
  int r = 53248 / stride;     // <= 52 KB stages: 16 rows at K=4096, 8 at K=12288
  if (r > 16) r = 16;
  if (r < 2) r = 2;
  return r;
}

template <int NCH>
static cudaError_t launch_nch(GemvArgs a, cudaStream_t st, bool pdl, int max_blocks) {
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv<NCH>, cudaFuncAttributeMaxDynamicSharedMemorySize, GT_CTA_SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int ru = a.rows_per_stage;
  int blocks = (a.total_units + ru - 1) / ru;
  if (blocks > max_blocks) blocks = max_blocks;
  const int min_blocks = (a.total_units + GT_RES_MAX - 1) / GT_RES_MAX;
  if (blocks < min_blocks) blocks = min_blocks;
  if (blocks < 1) blocks = 1;
  bool paired = false;
  for (int i = 0; i < a.nseg; ++i) paired |= a.seg[i].mode == GM_SILU_MUL;
  const size_t per_cta = (size_t)(a.total_units + blocks - 1) / blocks + 1;
  const size_t res_bytes = per_cta * (paired ? 2 : 1) * sizeof(long long);
  const size_t xs_bytes = (size_t)NCH * 4 * 32 * sizeof(uint2);
  const size_t stage_bytes = (size_t)a.rows_per_stage * a.stride;
  int stages = (int)(((long long)GT_CTA_SMEM - (long long)xs_bytes - (long long)res_bytes) / (long long)stage_bytes);
  if (stages > GT_MAX_STAGES) stages = GT_MAX_STAGES;
  if (stages < 2) return cudaErrorInvalidValue;
  a.stages = stages;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(GT_THREADS);
  cfg.dynamicSmemBytes = stages * stage_bytes + xs_bytes + res_bytes;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_gemv<NCH>, a);
}

cudaError_t launch_gemv(const GemvArgs &a_in, cudaStream_t st, bool pdl, int max_blocks) {
  GemvArgs a = a_in;
  a.rows_per_stage = gemv_rows_per_stage(a.stride);
  const int nch = (a.K + 1023) / 1024;
  switch (nch) {
    case 1: return launch_nch<1>(a, st, pdl, max_blocks);
    case 2: return launch_nch<2>(a, st, pdl, max_blocks);
    case 3: return launch_nch<3>(a, st, pdl, max_blocks);
    case 4: return launch_nch<4>(a, st, pdl, max_blocks);
    case 5: return launch_nch<5>(a, st, pdl, max_blocks);
    case 6: return launch_nch<6>(a, st, pdl, max_blocks);
    case 7: return launch_nch<7>(a, st, pdl, max_blocks);
    case 8: return launch_nch<8>(a, st, pdl, max_blocks);
    case 9: return launch_nch<9>(a, st, pdl, max_blocks);
    case 10: return launch_nch<10>(a, st, pdl, max_blocks);
    case 11: return launch_nch<11>(a, st, pdl, max_blocks);
    case 12: return launch_nch<12>(a, st, pdl, max_blocks);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace f5
