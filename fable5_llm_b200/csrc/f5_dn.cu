// Gated-DeltaNet decode step for one token (sm_100a), the vector part of
// ref/layer_fixed.py:1493-1580 deltanet_decode_fx between the in-projection
// GEMV (qkv16 / z16 / b / a) and the out-projection GEMV.
//
// One CTA per value head h (32 CTAs per sequence; 128 * NQ threads, thread
// t owns state column dv = t & 127).  The in-projection GEMV's epilogues already applied
// conv4 + SiLU per channel (the conv window is a 4-slot ring in HBM: slot T%4
// receives this step's input, the other three, oldest first, are the
// reference's conv state) and the gates beta / decay.  Per CTA:
//   l2norm of q and k; the recurrence on the int16
//   128x128 state (decay, kv_mem, delta, rank-1 update, clip16, o), staged
//   through shared memory; block-float shift k_h; the gated RMSNorm (float64
//   host-scale law or the integer EPS-NORM law) x norm_w x silu(z); output
//   clip16(on) for the out-projection's DYNQ8 prologue.
#include "f5_block.cuh"
#include "f5_dn.cuh"
#include "f5_dn_core.cuh"
#include "f5_kernels.cuh"
#include "f5_tma.cuh"

namespace f5 {

// One CTA of 128 * NQ threads per (value head, sequence): thread t owns
// state column t & 127 and the key rows of quarter t >> 7 (NQ = 1: all 128).
// Launched with NQ = 2: at 8 and 64 sequences, NQ = 1 and 2 measured the
// same and NQ = 4 was slower at 64.
//
// The per-sequence arguments of a batched launch are built member by member
// (no copy of a0 is modified): with nvcc 12.9 for sm_100a, advancing the
// first member of a local copy of the argument struct did not reach later
// reads of it.
template <int NQ>
__global__ void __launch_bounds__(128 * NQ) k_dn_step(const __grid_constant__ DnArgs a0, const DnBatch bs) {
  __shared__ __align__(128) int16_t s_sd[128 * 128];   // head state [dk][dv] -> decayed in place
  __shared__ int4 s_kq[128];
  __shared__ long long s_part[NQ > 1 ? NQ * 128 : 1];
  __shared__ long long red[32];
  __shared__ long long s_gate[4];             // beta, decay, rq, rk
  __shared__ int s_e[2];
  __shared__ __align__(8) uint64_t bar_s;

  const int h = blockIdx.x, t = threadIdx.x;
  const long long b = blockIdx.y;   // sequence of a batched launch
  DnArgs a;
  a.qkvc = a0.qkvc + b * bs.qkvc;
  a.beta = a0.beta + b * bs.gates;
  a.decay = a0.decay + b * bs.gates;
  a.z16 = a0.z16 + b * bs.z;
  a.norm_w = a0.norm_w;
  a.S = a0.S + b * bs.S;
  a.xslots = a0.xslots;
  a.in_tag_op1 = a0.in_tag_op1;
  a.out_tag_op1 = a0.out_tag_op1;
  a.on16 = a0.on16 + b * bs.on;
  a.kh_out = a0.kh_out ? a0.kh_out + b * bs.kh : nullptr;
  a.stats = a0.stats;
  a.err = a0.err;
  a.lkd = a0.lkd;
  a.vrep = a0.vrep;
  a.norm_mode = a0.norm_mode;
  // The head's 32 KB state does not depend on the previous kernel: start its
  // bulk copy into shared memory before the dependency wait.
  if (t == 0) {
    mbar_init(&bar_s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(&bar_s, 128 * 128 * 2);
    bulk_g2s(s_sd, a.S + (size_t)h * 128 * 128, 128 * 128 * 2, &bar_s);
  }
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const DnSmem sm = {s_sd, s_kq, NQ > 1 ? s_part : nullptr, red, s_gate, s_e};
  const BlockSync sy;
  long long qkv[3], zn[2];
  dn_head_pre<BlockSync, NQ>(sy, a, h, sm, qkv, zn);
  const bool got = mbar_wait(&bar_s, 0, 2000000000ull);
  if (sy.any(!got)) {
    // the state never arrived: flag it, leave S untouched, emit zeros (the
    // decision is block-uniform, so no thread is left at a barrier)
    if (t == 0) atomicOr(a.err, DERR_TIMEOUT);
    if (t < 128) a.on16[h * 128 + t] = 0;
    if (!got) mbar_wait(&bar_s, 0, 2000000000ull);
    return;
  }
  dn_head_rec<BlockSync, NQ>(sy, a, h, sm, qkv, zn);
}

// ntok consecutive tokens of ONE sequence (layer-major prompt prefill): the
// head's state is copied in once and stays in shared memory from token to
// token (dn_head_rec<KEEP>), token k's inputs / outputs at k times the
// DnBatch strides; S in HBM holds the state after every token.  One CTA per
// value head, as k_dn_step.
template <int NQ>
__global__ void __launch_bounds__(128 * NQ) k_dn_scan(const __grid_constant__ DnArgs a0, const DnBatch bs, int ntok) {
  __shared__ __align__(128) int16_t s_sd[128 * 128];
  __shared__ int4 s_kq[128];
  __shared__ long long s_part[NQ > 1 ? NQ * 128 : 1];
  __shared__ long long red[32];
  __shared__ long long s_gate[4];
  __shared__ int s_e[2];
  __shared__ __align__(8) uint64_t bar_s;

  const int h = blockIdx.x, t = threadIdx.x;
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (t == 0) {
    mbar_init(&bar_s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(&bar_s, 128 * 128 * 2);
    bulk_g2s(s_sd, a0.S + (size_t)h * 128 * 128, 128 * 128 * 2, &bar_s);
  }
  __syncthreads();   // the barrier is initialised before any thread waits on it
  const DnSmem sm = {s_sd, s_kq, NQ > 1 ? s_part : nullptr, red, s_gate, s_e};
  const BlockSync sy;
  const bool got = mbar_wait(&bar_s, 0, 2000000000ull);
  if (sy.any(!got)) {
    if (t == 0) atomicOr(a0.err, DERR_TIMEOUT);
    if (!got) mbar_wait(&bar_s, 0, 2000000000ull);
    return;
  }
  for (int k = 0; k < ntok; ++k) {
    DnArgs a;
    a.qkvc = a0.qkvc + k * bs.qkvc;
    a.beta = a0.beta + k * bs.gates;
    a.decay = a0.decay + k * bs.gates;
    a.z16 = a0.z16 + k * bs.z;
    a.norm_w = a0.norm_w;
    a.S = a0.S;
    a.xslots = a0.xslots;
    a.in_tag_op1 = a0.in_tag_op1;
    a.out_tag_op1 = a0.out_tag_op1;
    a.on16 = a0.on16 + k * bs.on;
    a.kh_out = a0.kh_out;
    a.stats = a0.stats;
    a.err = a0.err;
    a.lkd = a0.lkd;
    a.vrep = a0.vrep;
    a.norm_mode = a0.norm_mode;
    sy.sync();   // the previous token's readers of the shared scratch are done
    long long qkv[3], zn[2];
    dn_head_pre<BlockSync, NQ>(sy, a, h, sm, qkv, zn);
    dn_head_rec<BlockSync, NQ, true>(sy, a, h, sm, qkv, zn);
  }
}

cudaError_t launch_dn_scan(const DnArgs &a, const DnBatch &bs, int nheads, int ntok, cudaStream_t st) {
  k_dn_scan<2><<<nheads, 256, 0, st>>>(a, bs, ntok);
  return cudaGetLastError();
}

cudaError_t launch_dn_step(const DnArgs &a, int nheads, cudaStream_t st, bool pdl) {
  return launch_dn_step_b(a, DnBatch{}, nheads, 1, st, pdl);
}

cudaError_t launch_dn_step_b(const DnArgs &a, const DnBatch &bs, int nheads, int B, cudaStream_t st, bool pdl) {
  const int nq = 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nheads, B);
  cfg.blockDim = dim3(128 * nq);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  if (nq == 4) return cudaLaunchKernelEx(&cfg, k_dn_step<4>, a, bs);
  if (nq == 2) return cudaLaunchKernelEx(&cfg, k_dn_step<2>, a, bs);
  return cudaLaunchKernelEx(&cfg, k_dn_step<1>, a, bs);
}

}  // namespace f5
