// Persistent decode-step kernel: the whole 9B decode step (embedding row,
// every layer's GEMVs, DeltaNet and attention cores, the LM head and its
// argmax) as ONE cooperative launch over all SMs.  See f5_mega.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "f5_attn.cuh"
#include "f5_dn.cuh"
#include "f5_kernels.cuh"

namespace f5 {

enum MegaKind : int {
  MK_BEGIN = 0,   // x16 = emb[tok]; clear the argmax key, the attention sums and slots
  MK_GEMV = 1,    // one fused GEMV (same descriptor as k_gemv)
  MK_DN = 2,      // Gated-DeltaNet core, one value head per CTA
  MK_ATTN = 3,    // attention core, kv head x token chunk per CTA
};

struct MegaBegin {
  const int16_t *emb;         // [vocab][H]
  int16_t *x16;               // [H] plain residual (written back at the step's end)
  uint32_t *x16t;             // [H] tagged residual the step works on
  int res_row0, res_rows;     // this rank's rows of the 4096-row residual GEMVs
  int vocab, H;
  unsigned long long *key;    // LM-head argmax key
  uint4 *zero;                // attention accumulators, cleared every step
  int zero_n;                 // in uint4
};

struct MegaAttn {
  AttnArgs a;                 // same operands as the per-op attention kernel
  unsigned long long *slots;  // [2 phases][nkv][G / nkv CTAs][4 heads][2 words] marked values
  int32_t *gacc;              // [nq * HD] PV sums
  int in_tag_op1;             // dataflow tag of q|gate, k, v (tagged words)
};

// 16-byte aligned and sized: the kernel stages each descriptor in shared
// memory (bulk copy for the producer, vector loads for the consumers)
struct alignas(16) MegaOp {
  int kind;
  int bar;         // grid-barrier counter taken before the op (-1: the op's inputs are tagged)
  int pad[2];
  union {
    GemvArgs g;
    DnArgs d;
    MegaAttn at;
    MegaBegin b;
  };
};
static_assert(sizeof(MegaOp) % 16 == 0, "MegaOp is copied in 16-byte units");

struct MegaArgs {
  const MegaOp *ops;
  int nops;
  StepParams *params;
  unsigned *bars;   // [nbars] counters, zero at launch and zero again at exit
  int nbars;        // bars[nbars-2]: abort flag, bars[nbars-1]: final arrivals
  uint32_t *err;
  int advance;      // feed the argmax back as the next token (greedy loop)
  int dn_heads;     // CTAs [0, dn_heads) run one DeltaNet value head each
  int ns;           // ring stages (from mega_config)
  unsigned long long *trace;   // [G][nops][MEGA_TRACE_SLOTS] globaltimer marks (traced instance only)
  // row-sharded across nrank GPUs: the LM head's argmax keys are exchanged
  // through xkey ([F5_MAX_RANKS][2] marked words, in the twin allocation,
  // peers at + peer_delta[r])
  int nrank, rank;
  long long peer_delta[F5_MAX_RANKS];
  unsigned long long *xkey;
};

constexpr int MEGA_THREADS = 576;       // 16 consumer warps + producer warp + warp 17 (no role)
constexpr int MEGA_STAGE = 33792;       // ring stage: 16 rows of K=4096, 5 of K=12288
constexpr int MEGA_RES = 256;           // deferred per-CTA row results
constexpr int MEGA_SUB = 64;            // attention tokens per K/V shared-memory fill
// trace marks per (CTA, op): 0 start (after the grid barrier), 1 end,
// 2..6 op phases (GEMV: 2 prologue done, 3 rows done; DeltaNet: 2 l2norms,
// 3 state ready, 6 head done; attention: 2 q/k ready, 3 scores, 4 max,
// 5 sum, 6 PV sums), 7 arrival at the following grid barrier
constexpr int MEGA_TRACE_SLOTS = 8;

// Rows of one ring stage for a packed row stride.
inline int mega_rows_per_stage(int stride) {
  int r = MEGA_STAGE / stride;
  return r > 16 ? 16 : r;
}
// Grid (one CTA per SM) and dynamic shared memory of the persistent kernel
// for a given attention token chunk bound; error if it cannot be resident.
cudaError_t mega_config(int chunk_max, int *grid, size_t *smem, int *ns);
cudaError_t launch_mega(const MegaArgs &a, int grid, size_t smem, cudaStream_t st);
// The same step with per-op globaltimer marks written to a.trace (the traced
// instance, f5_mega_trace.cu); grid and smem from mega_config.
cudaError_t launch_mega_traced(const MegaArgs &a, int grid, size_t smem, cudaStream_t st);

}  // namespace f5
