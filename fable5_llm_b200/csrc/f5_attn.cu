// Full-attention decode step (sm_100a): the vector part of
// ref/layer_fixed.py:1383-1449 attn_decode_fx between the q|k|v GEMV and the
// o_proj GEMV, exactly integer.
//
// Grid: one thread-block cluster of ATT_SPLIT CTAs per query head; cluster
// rank c owns the token range [c*chunk, (c+1)*chunk) of the T+1 cached
// tokens (split-T, flash-decoding shape).  Integer sums are order-free, so
// the three cross-CTA reductions through distributed shared memory
// (max score, sum of exp, PV partial sums) are bit-exact for any split:
//   1. q/k RMSNorm(1+w) + partial RoPE, kv_quant of the new k and v
//      (every CTA recomputes them; the first CTA of the first head of each
//      KV group appends them to the int8 cache at slot T);
//   2. scores s = rshr(q.k8 * 2048, 15) -> Q16 (shift by QKV_F - ke - 16),
//      cluster max;
//   3. es = exp_neg_q(sc - max) (Q30), cluster sum, recip_q, p (Q15);
//   4. acc = sum_t rshr(p * v8, 15 - ve - QKV_F); cluster sum on rank 0,
//      times the sigmoid output gate -> int64 product for the o_proj prologue.
#include <climits>
#include <cooperative_groups.h>

#include "f5_attn.cuh"
#include "f5_block.cuh"
#include "f5_kernels.cuh"
#include "f5_tma.cuh"

namespace cg = cooperative_groups;

namespace f5 {

constexpr int ATT_THREADS = 256;

// RMSNorm(1+w) over the 256-dim head (ref/layer_fixed.py:1242-1278) followed
// by rope_fx on the first ROT dims (ref/layer_fixed.py:1340-1348).  x is this
// thread's element; returns the rotated, clipped value.
F5_DEV long long head_norm_rope(long long x, const int32_t *w, const int16_t *cs, int rot, long long *red,
                                long long *s_buf, int *s_int) {
  const int d = threadIdx.x;
  const long long ss = block_sum_ll(x * x, red);
  if (d == 0) {
    int64_t r; int e;
    rsqrt_q((uint64_t)(ss == 0 ? 1 : ss), 2 * QKV_F + 8, r, e);   // n = 256
    s_buf[0] = r;
    s_int[0] = e;
  }
  __syncthreads();
  const long long r = s_buf[0];
  const int e = s_int[0];
  long long y = clip(rshr(x * r, 30 - e), -(1ll << 32), (1ll << 32) - 1);
  const long long xn = clip16(rshr(y * ((long long)w[d] + (1 << 14)), 14));
  s_buf[8 + d] = xn;
  __syncthreads();
  long long out = xn;
  if (d < rot) {
    const int hh = rot >> 1;
    const long long rr = d < hh ? -s_buf[8 + d + hh] : s_buf[8 + d - hh];
    out = clip16(rshr(xn * cs[d] + rr * cs[64 + d], ROPE_F));
  }
  __syncthreads();
  return out;
}

// The per-sequence buffers of a batched launch are explicit local pointers
// (a is only read): with nvcc 12.9 for sm_100a, advancing the first member of
// a local copy of the argument struct did not reach later reads of it.
__global__ void __launch_bounds__(ATT_THREADS) k_attn(const __grid_constant__ AttnArgs a, const AttnBatch bs) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ long long red[32];
  __shared__ long long s_buf[8 + 256];
  __shared__ int s_int[8];
  __shared__ int32_t s_q[256];
  __shared__ __align__(16) int8_t s_k8[256];
  __shared__ __align__(16) int8_t s_v8[256];
  __shared__ int32_t s_acc[8][256];
  __shared__ long long s_part[4];                // [0] local max, [1] local sum
  __shared__ int32_t s_cacc[256];
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
  const int h = blockIdx.y;
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
  const int group = a.nq / a.nkv;
  const int kv = h / group;
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
  uint8_t *buf = dsm;                                          // [chunk][256]: K rows, then V rows
  int8_t *s_e8 = reinterpret_cast<int8_t *>(dsm + (size_t)a.chunk_max * 256);   // [chunk] exponents
  long long *s_sc = reinterpret_cast<long long *>(dsm + (size_t)a.chunk_max * 258);
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
      bulk_g2s(s_e8, ke + kv_row0, e_bytes, &bar_k);
    }
  }
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (!ok && c == 0 && d == 0 && h == 0) atomicOr(a.err, (uint32_t)DERR_KV_FULL);
  const int16_t *cs = a.rope + (size_t)pos * 128;

  // ---- 1. q, k norm + rope; kv_quant(k), kv_quant(v) ----
  const long long qv = head_norm_rope(qg16[h * 512 + d], a.q_norm, cs, a.rot, red, s_buf, s_int);
  s_q[d] = (int32_t)qv;
  const long long kn = head_norm_rope(k16[kv * 256 + d], a.k_norm, cs, a.rot, red, s_buf, s_int);
  const int ek = dynq8_e(block_max_ull(uabs(kn), reinterpret_cast<unsigned long long *>(red)));
  const long long vv = v16[kv * 256 + d];
  const int ev = dynq8_e(block_max_ull(uabs(vv), reinterpret_cast<unsigned long long *>(red)));
  const int8_t k8n = (int8_t)dynq8_apply(kn, ek), v8n = (int8_t)dynq8_apply(vv, ev);
  s_k8[d] = k8n;
  s_v8[d] = v8n;
  const int ke_new = ek - QKV_F, ve_new = ev - QKV_F;
  if (ok && c == 0 && (h % group) == 0) {
    const size_t row = ((size_t)kv * a.max_T + T) * 256;
    k8[row + d] = k8n;
    v8[row + d] = v8n;
    if (d == 0) {
      ke[(size_t)kv * a.max_T + T] = (int8_t)ke_new;
      ve[(size_t)kv * a.max_T + T] = (int8_t)ve_new;
    }
  }
  bool got = n_old == 0 || mbar_wait(&bar_k, 0, 2000000000ull);
  const bool kv_ok = !__syncthreads_or(!got);    // block-uniform
  if (!kv_ok && d == 0) atomicOr(a.err, (uint32_t)DERR_TIMEOUT);

  // ---- 2. scores over this CTA's token chunk (warp per token) ----
  int32_t qr[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) qr[j] = s_q[8 * lane + j];
  long long lmax = LLONG_MIN;
  for (int t = t0 + warp; t < t1; t += 8) {
    uint2 kw = make_uint2(0, 0);
    int ke = 0;
    if (ok && t == T) {
      kw = *reinterpret_cast<const uint2 *>(s_k8 + 8 * lane);
      ke = ke_new;
    } else if (kv_ok) {
      kw = *reinterpret_cast<const uint2 *>(buf + (size_t)(t - t0) * 256 + 8 * lane);
      ke = s_e8[t - t0];
    }
    int dot = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dot += qr[j] * (int)(int8_t)((kw.x >> (8 * j)) & 0xFF);
      dot += qr[4 + j] * (int)(int8_t)((kw.y >> (8 * j)) & 0xFF);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const long long sv = rshr((long long)dot * 2048, 15);   // SCALE_Q15 = round(2^15/sqrt(256))
    const long long sc = shift_to(sv, QKV_F - ke - 16);
    if (lane == 0) s_sc[t - t0] = sc;
    lmax = sc > lmax ? sc : lmax;
  }
  lmax = block_max_ll(lmax, red);   // ends with __syncthreads: the K rows are no longer read
  // V rows reuse the buffer; their copy overlaps the softmax phases
  if (d == 0 && n_old > 0 && got) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic reads before async writes
    mbar_expect_tx(&bar_v, row_bytes + e_bytes);
    bulk_g2s(buf, v8 + kv_row0 * 256, row_bytes, &bar_v);
    bulk_g2s(s_e8, ve + kv_row0, e_bytes, &bar_v);
  }
  if (d == 0) s_part[0] = lmax;
  cl.sync();
  long long mx = LLONG_MIN;
  for (int r = 0; r < nsplit; ++r) {
    const long long v = *cl.map_shared_rank(&s_part[0], r);
    mx = v > mx ? v : mx;
  }
  // ---- 3. exp, cluster sum, reciprocal ----
  long long lsum = 0;
  for (int i = d; i < t1 - t0; i += ATT_THREADS) {
    const long long x = s_sc[i] - mx;
    const long long es = exp_neg_q(x < 0 ? x : 0);
    s_sc[i] = es;
    lsum += es;
  }
  lsum = block_sum_ll(lsum, red);
  if (d == 0) s_part[1] = lsum;
  cl.sync();
  if (d == 0) {
    long long den = 0;
    for (int r = 0; r < nsplit; ++r) den += *cl.map_shared_rank(&s_part[1], r);
    int64_t rr; int re;
    recip_q((uint64_t)(den > 0 ? den : 1), 30, rr, re);
    s_buf[0] = rr;
    s_int[0] = re;
  }
  __syncthreads();
  const long long rcp = s_buf[0];
  const int psh = 30 - s_int[0] + 15;
  for (int i = d; i < t1 - t0; i += ATT_THREADS) s_sc[i] = clip(rshr(s_sc[i] * rcp, psh), 0, 1 << 15);
  got = n_old == 0 || !kv_ok || mbar_wait(&bar_v, 0, 2000000000ull);
  const bool v_ok = kv_ok && !__syncthreads_or(!got);
  if (kv_ok && !v_ok && d == 0) atomicOr(a.err, (uint32_t)DERR_TIMEOUT);

  // ---- 4. PV partial sums: warp w takes tokens t0+w, t0+w+8, ...; lane = 8 dims ----
  int32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int t = t0 + warp; t < t1; t += 8) {
    uint2 vw = make_uint2(0, 0);
    int ve = 0;
    if (ok && t == T) {
      vw = *reinterpret_cast<const uint2 *>(s_v8 + 8 * lane);
      ve = ve_new;
    } else if (v_ok) {
      vw = *reinterpret_cast<const uint2 *>(buf + (size_t)(t - t0) * 256 + 8 * lane);
      ve = s_e8[t - t0];
    }
    const int32_t p = (int32_t)s_sc[t - t0];
    const int sh = 15 - ve - QKV_F;                      // in [6, 15]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[j] += rshr32p(p * (int32_t)(int8_t)((vw.x >> (8 * j)) & 0xFF), sh);
      acc[4 + j] += rshr32p(p * (int32_t)(int8_t)((vw.y >> (8 * j)) & 0xFF), sh);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) s_acc[warp][8 * lane + j] = acc[j];
  __syncthreads();
  {
    int32_t sacc = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) sacc += s_acc[w][d];
    s_cacc[d] = sacc;
  }
  cl.sync();
  if (c == 0) {
    long long tot = 0;
    for (int r = 0; r < nsplit; ++r) tot += *cl.map_shared_rank(&s_cacc[d], r);
    // og = sigmoid_q(rshr(gate, QKV_F - 12)) = sigmoid_q(gate << 4)  (ref/layer_fixed.py:1436-1437)
    const long long og = sigmoid_q((long long)qg16[h * 512 + 256 + d] << (12 - QKV_F));
    prod[h * 256 + d] = tot * og;
  }
  // drain: no copy may still target this CTA's shared memory at exit
  if (d == 0 && n_old > 0 && !got) mbar_wait(&bar_v, 0, 2000000000ull);
  cl.sync();
}

cudaError_t launch_attn(const AttnArgs &a_in, cudaStream_t st, bool pdl) {
  return launch_attn_b(a_in, AttnBatch{}, 1, st, pdl);
}

cudaError_t launch_attn_b(const AttnArgs &a_in, const AttnBatch &bs, int B, cudaStream_t st, bool pdl) {
  const int nsplit = ATT_SPLIT;
  AttnArgs a = a_in;
  if (a.max_T % 16) return cudaErrorInvalidValue;
  a.chunk_max = (((a.max_T + nsplit - 1) / nsplit) + 15) & ~15;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsplit, a.nq, B);
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.dynamicSmemBytes = (size_t)a.chunk_max * (256 + 2 + 8);
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
  // static shared memory (~13 KB) + the K/V chunk: raise the per-kernel limit
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
