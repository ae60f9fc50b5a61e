// Gated-DeltaNet decode step for one token (sm_100a), the vector part of
// ref/layer_fixed.py:1493-1580 deltanet_decode_fx between the in-projection
// GEMV (qkv16 / z16 / b / a) and the out-projection GEMV.
//
// One CTA per value head h (32 CTAs x 128 threads; thread t owns state
// column dv = t).  Per CTA:
//   conv4 + SiLU of the 384 channels the head reads (q, k of key head h/2,
//   v of head h), with the conv window kept as a 4-slot ring in HBM (slot
//   T%4 receives this step's input; the other three, oldest first, are the
//   reference's conv state) -- no two CTAs read a slot another writes;
//   gates beta / decay; l2norm of q and k; the recurrence on the int16
//   128x128 state (decay, kv_mem, delta, rank-1 update, clip16, o), staged
//   through shared memory; block-float shift k_h; the gated RMSNorm (float64
//   host-scale law or the integer EPS-NORM law) x norm_w x silu(z); output
//   clip16(on) for the out-projection's DYNQ8 prologue.
#include "f5_block.cuh"
#include "f5_dn.cuh"
#include "f5_kernels.cuh"
#include "f5_tma.cuh"

namespace f5 {

constexpr int DN_THREADS = 128;

__global__ void __launch_bounds__(DN_THREADS) k_dn_step(const __grid_constant__ DnArgs a) {
  __shared__ __align__(128) int16_t s_sd[128 * 128];   // head state [dk][dv] -> decayed in place
  __shared__ int32_t s_qn[128], s_kn[128];
  __shared__ long long red[32];
  __shared__ long long s_gate[4];             // beta, decay, rq, rk
  __shared__ int s_e[2];
  __shared__ __align__(8) uint64_t bar_s;

  const int h = blockIdx.x, t = threadIdx.x;
  int16_t *S = a.S + (size_t)h * 128 * 128;
  // The head's 32 KB state does not depend on the previous kernel: start its
  // bulk copy into shared memory before the dependency wait.
  if (t == 0) {
    mbar_init(&bar_s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(&bar_s, 128 * 128 * 2);
    bulk_g2s(s_sd, S, 128 * 128 * 2, &bar_s);
  }
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int kh = h / a.vrep;
  const int T = *a.T;
  const int slot_new = T & 3;
  // ---- conv4 + SiLU (ref/layer_fixed.py:1515-1524) ----
  const int chans[3] = {kh * 128 + t, a.lkd + kh * 128 + t, 2 * a.lkd + h * 128 + t};
  long long qkv[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int c = chans[i];
    const int16_t *ring = a.conv + (size_t)c * 4;
    const int32_t *cw = a.conv_w + (size_t)c * 4;
    const long long xnew = a.qkv16[c];
    long long acc = 0;
#pragma unroll
    for (int j = 0; j < 3; ++j) acc += (long long)ring[(T + 1 + j) & 3] * cw[j];
    acc += xnew * cw[3];
    const long long pre = clip(rshr(acc, RS_F + CW_F - 12), -(1 << 20), (1 << 20) - 1);
    const long long co = clip16(silu_q(pre));
    qkv[i] = rshr(co, 12 - QKV_F);
  }
  // ---- gates (ref/layer_fixed.py:1531-1538) ----
  if (t == 0) {
    const long long beta = sigmoid_q(a.b16[h]);
    const long long sp = softplus_q((long long)a.a16[h] + a.dt_bias[h]);
    const long long g = -rshr((long long)a.A[h] * sp, 15 + 12 - 16);
    long long dec = rshr(exp_neg_q(g < 0 ? g : 0), 15);
    if (dec > 32767) dec = 32767;
    s_gate[0] = beta;
    s_gate[1] = dec;
  }
  // ---- l2norm of q and k (ref/layer_fixed.py:1322-1330, 1540-1543) ----
  const long long ssq = block_sum_ll(qkv[0] * qkv[0], red);
  const long long ssk = block_sum_ll(qkv[1] * qkv[1], red);
  if (t == 0) {
    int64_t r; int e;
    rsqrt_q((uint64_t)(ssq == 0 ? 1 : ssq), 2 * QKV_F, r, e);
    s_gate[2] = r; s_e[0] = e;
    rsqrt_q((uint64_t)(ssk == 0 ? 1 : ssk), 2 * QKV_F, r, e);
    s_gate[3] = r; s_e[1] = e;
  }
  __syncthreads();
  {
    const long long qn = clip16(rshr(qkv[0] * s_gate[2], QKV_F + 30 - s_e[0] - NRM_F));
    s_qn[t] = (int32_t)rshr(qn * 2896, 15);    // round(2^15 / sqrt(128)) = 2896
    s_kn[t] = (int32_t)clip16(rshr(qkv[1] * s_gate[3], QKV_F + 30 - s_e[1] - NRM_F));
  }
  // conv ring update: slot T%4 gets this step's pre-conv input; q/k channels
  // are shared by the VREP value heads of a key head -> written by the first
  if ((h % a.vrep) == 0) {
    a.conv[(size_t)chans[0] * 4 + slot_new] = a.qkv16[chans[0]];
    a.conv[(size_t)chans[1] * 4 + slot_new] = a.qkv16[chans[1]];
  }
  a.conv[(size_t)chans[2] * 4 + slot_new] = a.qkv16[chans[2]];
  __syncthreads();

  // ---- recurrence (ref/layer_fixed.py:1545-1571), column dv = t ----
  const bool got = mbar_wait(&bar_s, 0, 2000000000ull);
  if (__syncthreads_or(!got)) {
    // the state never arrived: flag it, leave S untouched, emit zeros (the
    // decision is block-uniform, so no thread is left at a barrier)
    if (t == 0) atomicOr(a.err, DERR_TIMEOUT);
    a.on16[h * 128 + t] = 0;
    if (!got) mbar_wait(&bar_s, 0, 2000000000ull);
    return;
  }
  const int decay = (int)s_gate[1];
  long long kvm = 0;
#pragma unroll 8
  for (int dk = 0; dk < 128; ++dk) {
    const int sd = rshr32p((int32_t)s_sd[dk * 128 + t] * decay, GAT_F);   // |S*decay| < 2^30
    s_sd[dk * 128 + t] = (int16_t)sd;
    kvm += (long long)sd * s_kn[dk];
  }
  kvm = rshr(kvm, NRM_F);
  const long long v_s = qkv[2] << (S_F - QKV_F);
  const long long delta = rshr((v_s - kvm) * s_gate[0], GAT_F);
  long long o = 0;
  int sat = 0;
#pragma unroll 8
  for (int dk = 0; dk < 128; ++dk) {
    long long sn = (long long)s_sd[dk * 128 + t] + rshr((long long)s_kn[dk] * delta, NRM_F);
    if (sn > 32767 || sn < -32767) ++sat;   // |Sh| > 32767 (ref/layer_fixed.py:1557)
    sn = clip16(sn);
    S[dk * 128 + t] = (int16_t)sn;
    o += sn * s_qn[dk];
  }
  o = rshr(o, NRM_F);
  if (a.stats && sat) atomicAdd(a.stats, (unsigned long long)sat);

  // ---- block floating k_h (ref/layer_fixed.py:470-486) ----
  const unsigned long long om = block_max_ull(uabs(o), reinterpret_cast<unsigned long long *>(red));
  const int kh_shift = bf_shift(om);
  const long long o16 = clip16(kh_shift >= 0 ? rshr(o, kh_shift) : (long long)((unsigned long long)o << (-kh_shift)));
  // ---- gated RMSNorm scale (ref/layer_fixed.py:509-546 or 694-781) ----
  long long m;
  if (a.norm_mode == 0) {
    // numpy int64 sum of o*o (wrapping modulo 2^64, order-free)
    const long long ss = (long long)block_sum_ull((unsigned long long)o * (unsigned long long)o,
                                                  reinterpret_cast<unsigned long long *>(red));
    m = dn_norm_scale(ss, kh_shift, 128);
  } else {
    const long long ss = block_sum_ll(o16 * o16, red);
    m = eps_norm_scale(ss, kh_shift, 7);
  }
  const long long tt = clip16(rshr(o16 * m, 15));
  const long long nh = clip16(rshr(tt * a.norm_w[t], 14));
  const long long zg = clip16(silu_q((long long)a.z16[h * 128 + t] << (12 - QKV_F)));
  a.on16[h * 128 + t] = (int16_t)clip16(rshr(nh * zg, 12));
  if (t == 0 && a.kh_out) a.kh_out[h] = kh_shift;
}

cudaError_t launch_dn_step(const DnArgs &a, int nheads, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nheads);
  cfg.blockDim = dim3(DN_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_dn_step, a);
}

}  // namespace f5
