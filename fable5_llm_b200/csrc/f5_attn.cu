// Full-attention decode step (sm_100a): the vector part of
// ref/layer_fixed.py:1383-1449 attn_decode_fx between the q|k|v GEMV and the
// o_proj GEMV, exactly integer.
//
// Grid: one thread-block cluster of ATT_SPLIT CTAs per KV head (and per
// sequence of a batched launch); cluster rank c owns the token range
// [c*chunk, (c+1)*chunk) of the T+1 cached tokens (split-T, flash-decoding
// shape) for all G = nq / nkv query heads of the KV group, so every cached
// K and V row is staged once.  Integer sums are order-free, so the three
// cross-CTA reductions through distributed shared memory (max score, sum of
// exp, PV partial sums) are bit-exact for any split:
//   1. q (G heads) / k RMSNorm(1+w) + partial RoPE, kv_quant of the new k
//      and v (the first CTA of each cluster appends them to the int8 cache
//      at slot T);
//   2. scores s = rshr(q.k8 * 2048, 15) -> Q16 (shift by QKV_F - ke - 16),
//      cluster max per head;
//   3. es = exp_neg_q(sc - max) (Q30), cluster sum, recip_q, p (Q15);
//   4. acc = sum_t rshr(p * v8, 15 - ve - QKV_F); cluster sum (rank g takes
//      head g), times the sigmoid output gate -> int64 product for the
//      o_proj prologue.
#include <climits>
#include <cooperative_groups.h>

#include "f5_attn.cuh"
#include "f5_block.cuh"
#include "f5_kernels.cuh"
#include "f5_tma.cuh"

namespace cg = cooperative_groups;

namespace f5 {

constexpr int ATT_THREADS = 256;
constexpr int ATT_GMAX = 4;   // query heads per KV head handled by one CTA

// Dynamic shared memory of one CTA: the K (then V) rows of its chunk, which
// later hold the four token phases' PV partial sums, the K and V exponents,
// and the scores / probabilities [chunk][ATT_GMAX] (int32).
F5_DEV_HOST_INLINE size_t att_buf_bytes(int chunk_max) {
  const size_t rows = (size_t)chunk_max * 256, parts = 4 * ATT_GMAX * 256 * 4;
  return rows > parts ? rows : parts;
}
F5_DEV_HOST_INLINE size_t att_smem_bytes(int chunk_max) {
  return att_buf_bytes(chunk_max) + (size_t)chunk_max * (2 + 4 * ATT_GMAX);
}

// RMSNorm(1+w) over the 256-dim head (ref/layer_fixed.py:1242-1278) of the
// G query heads and the key head at once (one reduction round for all sums
// of squares, the rsqrt of head i computed by thread i), followed by rope_fx
// on the first ROT dims (ref/layer_fixed.py:1340-1348).  x[i] is this
// thread's element of head i (slots 0..G-1: q heads, slot ATT_GMAX: the k
// head); on return x[i] is the rotated, clipped value.  s_x holds
// (ATT_GMAX+1) x 256 int32.
F5_DEV void heads_norm_rope(long long (&x)[ATT_GMAX + 1], int G, const int32_t *q_w, const int32_t *k_w,
                            const int16_t *cs, int rot, long long *red, int32_t *s_x, long long *s_r,
                            int *s_e) {
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
#pragma unroll
  for (int i = 0; i <= ATT_GMAX; ++i) {
    if (i >= G && i < ATT_GMAX) continue;
    long long s = x[i] * x[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp * (ATT_GMAX + 1) + i] = s;
  }
  __syncthreads();
  if (d < G || d == ATT_GMAX) {
    long long ss = 0;
    for (int w = 0; w < ATT_THREADS / 32; ++w) ss += red[w * (ATT_GMAX + 1) + d];
    int64_t r; int e;
    rsqrt_q((uint64_t)(ss == 0 ? 1 : ss), 2 * QKV_F + 8, r, e);   // n = 256
    s_r[d] = r;
    s_e[d] = e;
  }
  __syncthreads();
  const long long wq = (long long)q_w[d] + (1 << 14), wk = (long long)k_w[d] + (1 << 14);
#pragma unroll
  for (int i = 0; i <= ATT_GMAX; ++i) {
    if (i >= G && i < ATT_GMAX) continue;
    const long long y = clip(rshr(x[i] * s_r[i], 30 - s_e[i]), -(1ll << 32), (1ll << 32) - 1);
    x[i] = clip16(rshr(y * (i == ATT_GMAX ? wk : wq), 14));
    s_x[i * 256 + d] = (int32_t)x[i];
  }
  __syncthreads();
  if (d < rot) {
    const int hh = rot >> 1;
    const long long c0 = cs[d], s0 = cs[64 + d];
#pragma unroll
    for (int i = 0; i <= ATT_GMAX; ++i) {
      if (i >= G && i < ATT_GMAX) continue;
      const long long rr = d < hh ? -(long long)s_x[i * 256 + d + hh] : (long long)s_x[i * 256 + d - hh];
      x[i] = clip16(rshr(x[i] * c0 + rr * s0, ROPE_F));
    }
  }
}

// One CTA per (token chunk, KV head, sequence): the G query heads of the KV
// group share every K and V row this CTA stages, so each cached row crosses
// HBM once per step.  The per-sequence buffers of a batched launch are
// explicit local pointers (a is only read): with nvcc 12.9 for sm_100a,
// advancing the first member of a local copy of the argument struct did not
// reach later reads of it.
__global__ void __launch_bounds__(ATT_THREADS) k_attn(const __grid_constant__ AttnArgs a, const AttnBatch bs) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ long long red[64];
  __shared__ int32_t s_w[(ATT_GMAX + 1) * 256];   // normalised heads (rope partners), then PV sums [g][256]
  __shared__ __align__(16) int32_t s_q[ATT_GMAX][256];
  __shared__ __align__(16) int8_t s_k8[256];
  __shared__ __align__(16) int8_t s_v8[256];
  __shared__ long long s_part[2][ATT_GMAX];      // local max, local sum per head
  __shared__ long long s_r[ATT_GMAX + 1];
  __shared__ int s_e[ATT_GMAX + 1];
  __shared__ __align__(8) uint64_t bar_k, bar_v;

  // sequence blockIdx.z of a batched launch
  const long long sb = blockIdx.z;
  const int16_t *const qg16 = a.qg16 + sb * bs.qg;
  const int16_t *const k16 = a.k16 + sb * bs.kv16;
  const int16_t *const v16 = a.v16 + sb * bs.kv16;
  int8_t *const k8 = a.k8 + sb * bs.cache;
  int8_t *const v8 = a.v8 + sb * bs.cache;
  int8_t *const ke = a.ke + sb * bs.cache_e;
  int8_t *const ve = a.ve + sb * bs.cache_e;
  int64_t *const prod = a.prod + sb * bs.prod;
  const int *const Tp = a.T + sb * bs.params;
  const int *const posp = a.pos + sb * bs.params;
  cg::cluster_group cl = cg::this_cluster();
  const int c = (int)cl.block_rank();
  const int nsplit = (int)cl.num_blocks();
  const int kv = blockIdx.y;
  const int G = a.nq / a.nkv;   // 1..ATT_GMAX (checked by the launcher)
  const int h0 = kv * G;
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
  // T and pos are only written by the host or by the previous step's last
  // kernel, so they can be read before the dependency wait.
  const int T = *Tp;
  int pos = *posp;
  bool ok = T >= 0 && T < a.max_T;
  if (pos < 0 || pos >= a.max_pos) { ok = false; pos = 0; }
  const int Tn = ok ? T + 1 : max(0, min(T, a.max_T));   // tokens attended (incl. the new one)
  const int chunk = (((Tn + nsplit - 1) / nsplit) + 15) & ~15;
  const int t0 = c * chunk;
  const int t1 = min(t0 + chunk, Tn);
  const int Told = ok ? T : Tn;                  // cached rows (global memory)
  const int n_old = max(0, min(t1, Told) - t0);  // rows of this chunk already cached
  const uint32_t row_bytes = (uint32_t)n_old * 256, e_bytes = ((uint32_t)n_old + 15) & ~15u;
  const size_t bufb = att_buf_bytes(a.chunk_max);
  uint8_t *buf = dsm;                                               // K rows, then V rows, then PV partials
  int8_t *s_ke8 = reinterpret_cast<int8_t *>(dsm + bufb);           // [chunk] K exponents
  int8_t *s_ve8 = s_ke8 + a.chunk_max;                              // [chunk] V exponents
  int32_t *s_sc = reinterpret_cast<int32_t *>(s_ve8 + a.chunk_max);   // [chunk][ATT_GMAX]
  const size_t kv_row0 = (size_t)kv * a.max_T + t0;

  // cached K rows of this chunk do not depend on the previous kernel: copy
  // them into shared memory before the dependency wait
  if (d == 0) {
    mbar_init(&bar_k, 1);
    mbar_init(&bar_v, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (n_old > 0) {
      mbar_expect_tx(&bar_k, row_bytes + e_bytes);
      bulk_g2s(buf, k8 + kv_row0 * 256, row_bytes, &bar_k);
      bulk_g2s(s_ke8, ke + kv_row0, e_bytes, &bar_k);
    }
  }
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (!ok && c == 0 && d == 0 && kv == 0) atomicOr(a.err, (uint32_t)DERR_KV_FULL);
  const int16_t *cs = a.rope + (size_t)pos * 128;

  // ---- 1. q (G heads), k norm + rope; kv_quant(k), kv_quant(v) ----
  long long x[ATT_GMAX + 1];
#pragma unroll
  for (int g = 0; g < ATT_GMAX; ++g) x[g] = g < G ? (long long)qg16[(h0 + g) * 512 + d] : 0;
  x[ATT_GMAX] = k16[kv * 256 + d];
  const long long vv = v16[kv * 256 + d];
  heads_norm_rope(x, G, a.q_norm, a.k_norm, cs, a.rot, red, s_w, s_r, s_e);
#pragma unroll
  for (int g = 0; g < ATT_GMAX; ++g) s_q[g][d] = g < G ? (int32_t)x[g] : 0;
  const long long kn = x[ATT_GMAX];
  unsigned long long mk, mv;
  g_max2_ull(BlockSync{}, uabs(kn), uabs(vv), reinterpret_cast<unsigned long long *>(red), mk, mv);
  const int ek = dynq8_e(mk), ev = dynq8_e(mv);
  const int8_t k8n = (int8_t)dynq8_apply(kn, ek), v8n = (int8_t)dynq8_apply(vv, ev);
  s_k8[d] = k8n;
  s_v8[d] = v8n;
  const int ke_new = ek - QKV_F, ve_new = ev - QKV_F;
  if (ok && c == 0) {
    const size_t row = ((size_t)kv * a.max_T + T) * 256;
    k8[row + d] = k8n;
    v8[row + d] = v8n;
    if (d == 0) {
      ke[(size_t)kv * a.max_T + T] = (int8_t)ke_new;
      ve[(size_t)kv * a.max_T + T] = (int8_t)ve_new;
    }
  }
  bool got = n_old == 0 || mbar_wait(&bar_k, 0, 2000000000ull);
  const bool kv_ok = !__syncthreads_or(!got);    // block-uniform; also publishes s_q / s_k8 / s_v8
  if (!kv_ok && d == 0) atomicOr(a.err, (uint32_t)DERR_TIMEOUT);
  // exponent of token t's K row (zero rows when the copy failed)
  auto k_exp = [&](int t) -> int { return (ok && t == T) ? ke_new : (kv_ok ? (int)s_ke8[t - t0] : 0); };

  // ---- 2. scores over this CTA's token chunk (warp per token, lane = 8 dims, all G heads) ----
  int32_t qr[ATT_GMAX][8];
#pragma unroll
  for (int g = 0; g < ATT_GMAX; ++g) {
    const int4 lo = *reinterpret_cast<const int4 *>(&s_q[g][8 * lane]);
    const int4 hi = *reinterpret_cast<const int4 *>(&s_q[g][8 * lane + 4]);
    qr[g][0] = lo.x; qr[g][1] = lo.y; qr[g][2] = lo.z; qr[g][3] = lo.w;
    qr[g][4] = hi.x; qr[g][5] = hi.y; qr[g][6] = hi.z; qr[g][7] = hi.w;
  }
  const int gl = lane >> 3;   // head whose total this lane receives
  long long lmax = LLONG_MIN;
  for (int t = t0 + warp; t < t1; t += ATT_THREADS / 32) {
    uint2 kw = make_uint2(0, 0);
    if (ok && t == T) kw = *reinterpret_cast<const uint2 *>(s_k8 + 8 * lane);
    else if (kv_ok) kw = *reinterpret_cast<const uint2 *>(buf + (size_t)(t - t0) * 256 + 8 * lane);
    int kb[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      kb[j] = (int)(int8_t)((kw.x >> (8 * j)) & 0xFF);
      kb[4 + j] = (int)(int8_t)((kw.y >> (8 * j)) & 0xFF);
    }
    int dot[4];
#pragma unroll
    for (int g = 0; g < ATT_GMAX; ++g) {
      int s = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) s += qr[g][j] * kb[j];
      dot[g] = s;
    }
    const int tot = warp_sum4_i32(dot);
    const int32_t sv = (int32_t)rshr((long long)tot * 2048, 15);   // SCALE_Q15 = round(2^15/sqrt(256))
    if ((lane & 7) == 0) s_sc[(t - t0) * ATT_GMAX + gl] = sv;
    const long long sc = shift_to(sv, QKV_F - k_exp(t) - 16);
    lmax = sc > lmax ? sc : lmax;
  }
  if ((lane & 7) == 0) red[warp * ATT_GMAX + gl] = lmax;
  __syncthreads();   // the K rows are no longer read
  // V rows reuse the buffer; their copy overlaps the softmax phases
  if (d == 0 && n_old > 0 && kv_ok) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic reads before async writes
    mbar_expect_tx(&bar_v, row_bytes + e_bytes);
    bulk_g2s(buf, v8 + kv_row0 * 256, row_bytes, &bar_v);
    bulk_g2s(s_ve8, ve + kv_row0, e_bytes, &bar_v);
  }
  if (d < G) {
    long long m = red[d];
    for (int w = 1; w < ATT_THREADS / 32; ++w) m = red[w * ATT_GMAX + d] > m ? red[w * ATT_GMAX + d] : m;
    s_part[0][d] = m;
  }
  cl.sync();
  // ---- 3. exp, cluster sum, reciprocal (thread d works on head d % 4) ----
  const int gd = d & (ATT_GMAX - 1);
  long long mx = LLONG_MIN;
  for (int r = 0; r < nsplit; ++r) {
    const long long v = gd < G ? *cl.map_shared_rank(&s_part[0][gd], r) : 0;
    mx = v > mx ? v : mx;
  }
  const int n = t1 - t0;
  long long lsum = 0;
  if (gd < G) {
    for (int i = d; i < n * ATT_GMAX; i += ATT_THREADS) {
      const int t = t0 + i / ATT_GMAX;
      const long long xs = shift_to(s_sc[i], QKV_F - k_exp(t) - 16) - mx;
      const long long es = exp_neg_q(xs < 0 ? xs : 0);   // Q30, <= 2^30
      s_sc[i] = (int32_t)es;
      lsum += es;
    }
  }
#pragma unroll
  for (int o = 16; o >= ATT_GMAX; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
  if (lane < ATT_GMAX) red[warp * ATT_GMAX + lane] = lsum;
  __syncthreads();
  if (d < G) {
    long long s = 0;
    for (int w = 0; w < ATT_THREADS / 32; ++w) s += red[w * ATT_GMAX + d];
    s_part[1][d] = s;
  }
  cl.sync();
  if (d < G) {
    long long den = 0;
    for (int r = 0; r < nsplit; ++r) den += *cl.map_shared_rank(&s_part[1][d], r);
    int64_t rr; int re;
    recip_q((uint64_t)(den > 0 ? den : 1), 30, rr, re);
    s_r[d] = rr;
    s_e[d] = re;
  }
  __syncthreads();
  if (gd < G) {
    const long long rcp = s_r[gd];
    const int psh = 30 - s_e[gd] + 15;
    for (int i = d; i < n * ATT_GMAX; i += ATT_THREADS) s_sc[i] = (int32_t)clip(rshr((long long)s_sc[i] * rcp, psh), 0, 1 << 15);
  }
  got = n_old == 0 || !kv_ok || mbar_wait(&bar_v, 0, 2000000000ull);
  const bool v_ok = kv_ok && !__syncthreads_or(!got);
  if (kv_ok && !v_ok && d == 0) atomicOr(a.err, (uint32_t)DERR_TIMEOUT);

  // ---- 4. PV partial sums: thread = 4 dims (dq) x token phase ph, all G heads ----
  const int dq = d & 63, ph = d >> 6;
  int32_t acc[ATT_GMAX][4];
#pragma unroll
  for (int g = 0; g < ATT_GMAX; ++g)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[g][j] = 0;
  for (int t = t0 + ph; t < t1; t += 4) {
    uint32_t vw = 0;
    int vex = 0;
    if (ok && t == T) {
      vw = *reinterpret_cast<const uint32_t *>(s_v8 + 4 * dq);
      vex = ve_new;
    } else if (v_ok) {
      vw = *reinterpret_cast<const uint32_t *>(buf + (size_t)(t - t0) * 256 + 4 * dq);
      vex = s_ve8[t - t0];
    }
    const int4 p4 = *reinterpret_cast<const int4 *>(s_sc + (t - t0) * ATT_GMAX);
    const int p[4] = {p4.x, p4.y, p4.z, p4.w};
    const int sh = 15 - vex - QKV_F;                      // in [6, 15]
    const int32_t add = 1 << (sh - 1);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // rshr32p(p * v, sh) with p >= 0: sign(v) * ((p * |v| + add) >> sh)
      const int32_t v = (int32_t)(int8_t)((vw >> (8 * j)) & 0xFF);
      const int32_t av = v < 0 ? -v : v, sg = v >> 31;
#pragma unroll
      for (int g = 0; g < ATT_GMAX; ++g) {
        const int32_t r = (p[g] * av + add) >> sh;
        acc[g][j] += (r ^ sg) - sg;
      }
    }
  }
  // drain: no copy may still target this CTA's shared memory past this point
  if (d == 0 && n_old > 0 && !kv_ok) mbar_wait(&bar_k, 0, 2000000000ull);
  if (d == 0 && n_old > 0 && kv_ok && !got) mbar_wait(&bar_v, 0, 2000000000ull);
  __syncthreads();   // the V rows are no longer read: the buffer takes the partials
  int32_t *part = reinterpret_cast<int32_t *>(buf);   // [ph][g][256]
#pragma unroll
  for (int g = 0; g < ATT_GMAX; ++g)
    *reinterpret_cast<int4 *>(part + (ph * ATT_GMAX + g) * 256 + 4 * dq) =
        make_int4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
  __syncthreads();
#pragma unroll
  for (int g = 0; g < ATT_GMAX; ++g) {
    if (g >= G) break;
    int32_t s = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) s += part[(q * ATT_GMAX + g) * 256 + d];
    s_w[g * 256 + d] = s;
  }
  cl.sync();
  // rank g sums head g over the cluster (rank c also takes heads c + nsplit, ...)
  for (int g = c; g < G; g += nsplit) {
    long long tot = 0;
    for (int r = 0; r < nsplit; ++r) tot += *cl.map_shared_rank(&s_w[g * 256 + d], r);
    // og = sigmoid_q(rshr(gate, QKV_F - 12)) = sigmoid_q(gate << 4)  (ref/layer_fixed.py:1436-1437)
    const long long og = sigmoid_q((long long)qg16[(h0 + g) * 512 + 256 + d] << (12 - QKV_F));
    prod[(h0 + g) * 256 + d] = tot * og;
  }
  cl.sync();
}

cudaError_t launch_attn(const AttnArgs &a_in, cudaStream_t st, bool pdl) {
  return launch_attn_b(a_in, AttnBatch{}, 1, st, pdl);
}

cudaError_t launch_attn_b(const AttnArgs &a_in, const AttnBatch &bs, int B, cudaStream_t st, bool pdl) {
  const int nsplit = ATT_SPLIT;
  AttnArgs a = a_in;
  if (a.max_T % 16 || a.nkv <= 0 || a.nq % a.nkv || a.nq / a.nkv > ATT_GMAX) return cudaErrorInvalidValue;
  a.chunk_max = (((a.max_T + nsplit - 1) / nsplit) + 15) & ~15;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsplit, a.nkv, B);
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.dynamicSmemBytes = att_smem_bytes(a.chunk_max);
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = nsplit;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  // static shared memory (~9 KB) + the K/V chunk: raise the per-kernel limit
  // whenever the sum may pass the 48 KB default, not only when the chunk does
  static int attr_bytes = 0;
  if ((int)cfg.dynamicSmemBytes > attr_bytes) {
    cudaError_t e = cudaFuncSetAttribute(k_attn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)cfg.dynamicSmemBytes);
    if (e != cudaSuccess) return e;
    attr_bytes = (int)cfg.dynamicSmemBytes;
  }
  return cudaLaunchKernelEx(&cfg, k_attn, a, bs);
}

}  // namespace f5
