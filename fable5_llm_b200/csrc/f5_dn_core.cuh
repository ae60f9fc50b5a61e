// Device core of the Gated-DeltaNet decode step for one value head
// (ref/layer_fixed.py:1522-1580, after the in-projection epilogues' conv and
// gates), shared by the per-op kernel k_dn_step and the persistent kernel.  A group of NQ*128 threads runs one head:
// thread t owns value column dv = t & 127 and, in the recurrence, the state
// rows dk in quarter q = t >> 7 (NQ = 1: all 128 rows).  Integer sums are
// order-free, so splitting the dk reductions across threads is exact.
// Activations written by other CTAs of the same kernel are read at L2
// (__ldcg): the persistent kernel separates producer and consumer CTAs by a
// grid barrier, and L1 is not coherent across CTAs.
#pragma once
#include "f5_block.cuh"
#include "f5_dn.cuh"
#include "f5_kernels.cuh"

namespace f5 {

// State layout of a head, in HBM and in shared memory: [dv / 32][dk][dv % 32]
// (four 8 KB column quarters, each contiguous: one bulk copy per quarter).
F5_DEV int sidx(int dk, int dv) { return ((dv >> 5) << 12) | (dk << 5) | (dv & 31); }

struct DnSmem {
  int16_t *sd;      // [128*128] head state, sidx layout (decayed in place)
  int4 *kq;         // [128] per key row dk: kn, |kn|, sign(kn) (0 / -1), qn
  long long *part;  // [NQ*128] partial sums of the split recurrence
  long long *red;   // [32]
  long long *gate;  // [4] beta, decay, rq, rk
  int *e;           // [2]
};

// Inputs of the head and the l2norms of q and k (ref/layer_fixed.py:
// 1522-1543).  Conv4+SiLU and the gates were applied by the in-projection's
// epilogues, so every input is issued in one round of loads: post-conv q, k
// (key head h / vrep) and v, z, norm_w, beta, decay.  qkv[] / zn[] hold this
// column's q, k, v and z, norm_w (valid for q == 0).
template <class SY, int NQ>
F5_DEV void dn_head_pre(const SY &sy, const DnArgs &a, int h, const DnSmem &sm, long long (&qkv)[3],
                        long long (&zn)[2]) {
  const int t = sy.tid(), dv = t & 127, q = t >> 7;
  const int kh = h / a.vrep;
  qkv[0] = qkv[1] = qkv[2] = 0;
  zn[0] = zn[1] = 0;
  if (q == 0) {
    qkv[0] = __ldcg(a.qkvc + kh * 128 + dv);
    qkv[1] = __ldcg(a.qkvc + a.lkd + kh * 128 + dv);
    qkv[2] = __ldcg(a.qkvc + 2 * a.lkd + h * 128 + dv);
    zn[0] = __ldcg(a.z16 + h * 128 + dv);
    zn[1] = __ldcg(a.norm_w + dv);
  }
  if (t == 0) {
    sm.gate[0] = __ldcg(a.beta + h);
    sm.gate[1] = __ldcg(a.decay + h);
  }
  const long long ssq = g_sum_ll(sy, qkv[0] * qkv[0], sm.red);
  const long long ssk = g_sum_ll(sy, qkv[1] * qkv[1], sm.red);
  if (t == 0) {   // ref/layer_fixed.py:1322-1330
    int64_t r; int e;
    rsqrt_q((uint64_t)(ssq == 0 ? 1 : ssq), 2 * QKV_F, r, e);
    sm.gate[2] = r; sm.e[0] = e;
  } else if (t == 32) {
    int64_t r; int e;
    rsqrt_q((uint64_t)(ssk == 0 ? 1 : ssk), 2 * QKV_F, r, e);
    sm.gate[3] = r; sm.e[1] = e;
  }
  sy.sync();
  if (q == 0) {
    const long long qn = clip16(rshr(qkv[0] * sm.gate[2], QKV_F + 30 - sm.e[0] - NRM_F));
    const int32_t kn = clip16(rshr(qkv[1] * sm.gate[3], QKV_F + 30 - sm.e[1] - NRM_F));
    sm.kq[dv] = make_int4(kn, kn < 0 ? -kn : kn, kn >> 31,
                          (int32_t)rshr(qn * 2896, 15));    // round(2^15 / sqrt(128)) = 2896
  }
  sy.sync();
}

// recurrence, block-float shift, gated norm, x silu(z)  (ref/layer_fixed.py:
// 1545-1580).  sm.sd must hold the head's state.  KEEP: the new state also
// stays in sm.sd (each thread rewrites the entries it read), for a next
// token of the same sequence.
template <class SY, int NQ, bool KEEP = false>
F5_DEV void dn_head_rec(const SY &sy, const DnArgs &a, int h, const DnSmem &sm, const long long (&qkv)[3],
                        const long long (&zn)[2]) {
  const int t = sy.tid(), dv = t & 127, q = t >> 7;
  constexpr int RQ = 128 / NQ;
  int16_t *S = a.S + (size_t)h * 128 * 128;
  const int decay = (int)sm.gate[1];
  long long kvm = 0;
#pragma unroll 8
  for (int dk = q * RQ; dk < (q + 1) * RQ; ++dk) {
    const int sd = rshr32p((int32_t)sm.sd[sidx(dk, dv)] * decay, GAT_F);   // |S*decay| < 2^30
    sm.sd[sidx(dk, dv)] = (int16_t)sd;
    kvm += (long long)sd * sm.kq[dk].x;
  }
  if (NQ > 1) {
    sm.part[q * 128 + dv] = kvm;
    sy.sync();
    kvm = 0;
#pragma unroll
    for (int i = 0; i < NQ; ++i) kvm += sm.part[i * 128 + dv];
    sy.sync();
  }
  kvm = rshr(kvm, NRM_F);
  const long long v_col = NQ > 1 ? 0 : qkv[2];
  long long delta;
  if (NQ > 1) {
    if (q == 0) sm.part[dv] = rshr(((qkv[2] << (S_F - QKV_F)) - kvm) * sm.gate[0], GAT_F);
    sy.sync();
    delta = sm.part[dv];
    sy.sync();
  } else {
    delta = rshr(((v_col << (S_F - QKV_F)) - kvm) * sm.gate[0], GAT_F);
  }
  long long o = 0;
  int sat = 0;
  const unsigned long long dabs = uabs(delta);
  if (dabs < (1ull << 24)) {
    // |delta| < 2^24 (always, for beta <= 2^15): the rank-1 term in 32-bit
    // integers.  rshr(kn * delta, NRM_F) = sign(kn * delta) *
    // floor((|kn| |delta| + 2^(NRM_F-1)) / 2^NRM_F), and with |delta| =
    // dh 2^NRM_F + dl that floor is |kn| dh + ((|kn| dl + 2^(NRM_F-1)) >> NRM_F).
    const int32_t dh = (int32_t)(dabs >> NRM_F), dl = (int32_t)(dabs & ((1u << NRM_F) - 1));
    const int32_t sdl = delta < 0 ? -1 : 0;
#pragma unroll
    for (int c0 = q * RQ; c0 < (q + 1) * RQ; c0 += 16) {
      int32_t oc = 0;   // 16 terms of |sn * qn| <= 2^15 * 2896 stay below 2^31
#pragma unroll
      for (int dk = c0; dk < c0 + 16; ++dk) {
        const int4 kq = sm.kq[dk];
        const int32_t sg = kq.z ^ sdl;
        const int32_t r = kq.y * dh + ((kq.y * dl + (1 << (NRM_F - 1))) >> NRM_F);
        int32_t sn = (int32_t)sm.sd[sidx(dk, dv)] + ((r ^ sg) - sg);
        sat += (uint32_t)(sn + 32767) > 65534u;   // |Sh| > 32767 (ref/layer_fixed.py:1557)
        sn = min(max(sn, -32768), 32767);
        S[sidx(dk, dv)] = (int16_t)sn;
        if (KEEP) sm.sd[sidx(dk, dv)] = (int16_t)sn;
        oc += sn * kq.w;
      }
      o += oc;
    }
  } else {
#pragma unroll 8
    for (int dk = q * RQ; dk < (q + 1) * RQ; ++dk) {
      const int4 kq = sm.kq[dk];
      long long sn = (long long)sm.sd[sidx(dk, dv)] + rshr((long long)kq.x * delta, NRM_F);
      if (sn > 32767 || sn < -32767) ++sat;   // |Sh| > 32767 (ref/layer_fixed.py:1557)
      sn = clip16(sn);
      S[sidx(dk, dv)] = (int16_t)sn;
      if (KEEP) sm.sd[sidx(dk, dv)] = (int16_t)sn;
      o += sn * kq.w;
    }
  }
  if (a.stats && sat) atomicAdd(a.stats, (unsigned long long)sat);
  if (NQ > 1) {
    sm.part[q * 128 + dv] = o;
    sy.sync();
    o = 0;
#pragma unroll
    for (int i = 0; i < NQ; ++i) o += sm.part[i * 128 + dv];
    sy.sync();
  }
  o = rshr(o, NRM_F);
  if (q != 0) o = 0;   // one contribution per column to the head reductions
  // ---- block floating k_h (ref/layer_fixed.py:470-486) ----
  const unsigned long long om = g_max_ull(sy, uabs(o), reinterpret_cast<unsigned long long *>(sm.red));
  const int kh_shift = bf_shift(om);
  const long long o16 = clip16(kh_shift >= 0 ? rshr(o, kh_shift) : (long long)((unsigned long long)o << (-kh_shift)));
  // ---- gated RMSNorm scale (ref/layer_fixed.py:509-546 or 694-781) ----
  long long m;
  if (a.norm_mode == 0) {
    // numpy int64 sum of o*o (wrapping modulo 2^64, order-free)
    const long long ss = (long long)g_sum_ull(sy, (unsigned long long)o * (unsigned long long)o,
                                              reinterpret_cast<unsigned long long *>(sm.red));
    m = dn_norm_scale(ss, kh_shift, 128);
  } else {
    const long long ss = g_sum_ll(sy, o16 * o16, sm.red);
    m = eps_norm_scale(ss, kh_shift, 7);
  }
  if (q == 0) {
    const long long tt = clip16(rshr(o16 * m, 15));
    const long long nh = clip16(rshr(tt * zn[1], 14));
    const long long zg = clip16(silu_q(zn[0] << (12 - QKV_F)));
    a.on16[h * 128 + dv] = (int16_t)clip16(rshr(nh * zg, 12));
    if (dv == 0 && a.kh_out) a.kh_out[h] = kh_shift;
  }
}

}  // namespace f5
