// Attention decode kernel arguments (see f5_attn.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace f5 {

constexpr int ATT_SPLIT = 8;   // CTAs per query head (one portable cluster)

struct AttnArgs {
  const int16_t *qg16;    // [NQ][2*HD] q | gate per head (clip16, Q.QKV_F)
  const int16_t *k16;     // [NKV][HD]
  const int16_t *v16;     // [NKV][HD]
  const int32_t *q_norm;  // [HD] Q14 (zero-centred, 1+w)
  const int32_t *k_norm;  // [HD]
  const int16_t *rope;    // [max_pos][128]: cos Q15 [64] | sin Q15 [64]
  int8_t *k8, *ke;        // [NKV][max_T][HD], [NKV][max_T]
  int8_t *v8, *ve;
  int64_t *prod;          // [NQ*HD] out: acc * sigmoid(gate) (int64)
  const int *T;           // tokens already cached (new token goes to slot T)
  const int *pos;         // rope position of this token
  uint32_t *err;
  int max_T, max_pos;    // max_T a multiple of 16
  int chunk_max;          // set by launch_attn
  int nq, nkv, rot;
};

// Batched launch (B independent sequences, blockIdx.z = sequence): element
// strides between consecutive sequences' buffers (params: ints between the
// sequences' T / pos words)
struct AttnBatch {
  long long qg, kv16, cache, cache_e, prod, params;
};

cudaError_t launch_attn(const AttnArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_attn_b(const AttnArgs &a, const AttnBatch &bs, int B, cudaStream_t st, bool pdl);

}  // namespace f5
