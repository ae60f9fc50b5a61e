// DeltaNet step kernel arguments (see f5_dn.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace f5 {

// The in-projection GEMV's epilogues have already applied conv4+SiLU per
// channel (GM_CONV: post-conv q|k|v, conv ring advanced) and the per-head
// gates (GM_GATE_B / GM_GATE_A), so the step starts at the l2norms.
struct DnArgs {
  const int16_t *qkvc;    // [CONV_DIM] post-conv q | k | v (Q.QKV_F)
  const int32_t *beta;    // [LNH] sigmoid(b) (Q15)
  const int32_t *decay;   // [LNH] exp(g) (Q15)
  const int16_t *z16;     // [LVD] (Q.QKV_F)
  const int32_t *norm_w;  // [LDV] (Q14)
  int16_t *S;             // [LNH][4][LDK][32] int16 state (Q.S_F): head, dv / 32, dk, dv % 32
  unsigned long long *xslots;  // persistent kernel: [LNH][128][2] marked o values (zeroed per step)
  int in_tag_op1, out_tag_op1; // persistent kernel: dataflow tags of qkvc/z/beta/decay and of on16
  int16_t *on16;          // [LVD] out: clip16(on), Q.DN_NORM_F
  int *kh_out;            // optional [LNH] block-float shifts k_h
  unsigned long long *stats;  // optional: state saturation count
  uint32_t *err;          // device error word (DERR_TIMEOUT)
  int lkd;                // key channels (LNKH * LDK)
  int vrep;               // value heads per key head
  int norm_mode;          // 0 float64 host-scale law, 1 integer EPS-NORM
};

// Batched launch (B independent sequences, blockIdx.y = sequence): element
// strides between consecutive sequences' buffers
struct DnBatch {
  long long qkvc, gates, z, S, on, kh;
};

cudaError_t launch_dn_step(const DnArgs &a, int nheads, cudaStream_t st, bool pdl);
cudaError_t launch_dn_step_b(const DnArgs &a, const DnBatch &bs, int nheads, int B, cudaStream_t st, bool pdl);
// ntok consecutive tokens of one sequence (token k's inputs / outputs at k
// times bs's strides; one state)
cudaError_t launch_dn_scan(const DnArgs &a, const DnBatch &bs, int nheads, int ntok, cudaStream_t st);

}  // namespace f5
