// DeltaNet step kernel arguments (see f5_dn.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace f5 {

struct DnArgs {
  const int16_t *qkv16;   // [CONV_DIM] pre-conv in_qkv output (clip16, Q.RS_F)
  const int16_t *z16;     // [LVD] (Q.QKV_F)
  const int16_t *b16;     // [LNH] (Q12)
  const int16_t *a16;     // [LNH] (Q12)
  int16_t *conv;          // [CONV_DIM][4] ring of pre-conv inputs
  const int32_t *conv_w;  // [CONV_DIM][4] (Q.CW_F)
  const int32_t *dt_bias; // [LNH] (Q12)
  const int32_t *A;       // [LNH] (Q15, port-saturated)
  const int32_t *norm_w;  // [LDV] (Q14)
  int16_t *S;             // [LNH][LDK][LDV] int16 state (Q.S_F)
  int16_t *on16;          // [LVD] out: clip16(on), Q.DN_NORM_F
  const int *T;           // tokens already in the window (ring slot = T % 4)
  int *kh_out;            // optional [LNH] block-float shifts k_h
  unsigned long long *stats;  // optional: state saturation count
  uint32_t *err;          // device error word (DERR_TIMEOUT)
  int lkd;                // key channels (LNKH * LDK)
  int vrep;               // value heads per key head
  int norm_mode;          // 0 float64 host-scale law, 1 integer EPS-NORM
};

cudaError_t launch_dn_step(const DnArgs &a, int nheads, cudaStream_t st, bool pdl);

}  // namespace f5
