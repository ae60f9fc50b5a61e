// Kernel argument structs and host-side launchers of the sm_100a decode path.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define F5_DEV_HOST_INLINE __host__ __device__ __forceinline__

namespace f5 {

// ---- device error word bits (set by kernels, read by the host) ----
enum : uint32_t {
  DERR_Y32_OVERFLOW = 1u << 0,   // |y32| >= 2^31 (ref/w4a8_ref.py:288 assert)
  DERR_TIMEOUT = 1u << 1,        // a bounded device wait gave up
  DERR_KV_FULL = 1u << 2,        // KV append beyond max_T
  DERR_RANGE = 1u << 3,          // an input outside a documented range
};

// ---- device-resident step parameters (read by the decode step's kernels) ----
struct StepParams {
  int tok;        // input token of this step
  int pos;        // RoPE position of this step
  int T;          // tokens already in every layer's cache / conv window
  int next_tok;   // argmax of this step (first max wins)
  int max_val;    // its y32 logit
  uint32_t err;   // device error bits (DERR_*)
  int steps;      // steps completed since reset
  int launch;     // persistent-kernel launches since reset (dataflow tag epoch)
};

// ---- dataflow tags of the persistent kernel ----
// An activation word is (tag << 16) | uint16 value, tag = epoch << 8 | op:
// epoch = 1 + launch % 255 (never 0, so zeroed buffers never match), op =
// the writer's index in the step's op list (< 256).  A reader polls its
// input words until every tag matches the expected writer: the word carries
// its own readiness, so no grid barrier is needed between the two ops.
F5_DEV_HOST_INLINE uint32_t mega_epoch(int launch) { return 1u + (uint32_t)(launch % 255); }

// ---- quantized activation vector (DYNQ8 output, ref/fixedpoint.py:24-33) ----
// x8 lives in its own buffer; meta[0] = e_x, meta[1] = in_f (fraction bits
// of the int16 vector that was quantized; consumed by matvec_to's shift).
struct XQ {
  int8_t *x8;
  int *meta;
};

// ---- GEMV (batch-1 W4A8 matvec over packed DDR rows) ----
enum GemvMode : int {
  GM_Y32 = 0,       // out int32[row] = y32
  GM_TO16 = 1,      // out int16[row] = clip16(matvec_to shift)
  GM_TO64 = 2,      // out int64[row] = matvec_to shift
  GM_RESID = 3,     // out int16[row] = clip16(out[row] + clip16(shift))
  GM_SILU_MUL = 4,  // paired gate/up rows -> clip16(rshr(silu(g) * u, 12))
  GM_ARGMAX = 5,    // running (max y32, lowest row) key
  // DeltaNet in-projection epilogues (ref/layer_fixed.py:1511-1538): the
  // per-channel / per-head vector work that does not need the whole head
  GM_CONV = 6,      // out int16 = v = clip16(shift) (pre-conv, Q.RS_F); aux_out int16 =
                    // conv4+SiLU of the channel over its ring (Q.QKV_F); ring[T % 4] = v
  GM_GATE_B = 7,    // out int16 = v (Q12); aux_out int32 = beta = sigmoid_q(v)
  GM_GATE_A = 8,    // out int16 = v (Q12); aux_out int32 = decay of softplus(v + dt_bias) * A
};

constexpr int GEMV_MAX_SEG = 4;
constexpr int F5_MAX_RANKS = 8;

// How a GEMV CTA obtains its quantized input x8 (+ e_x, in_f).  Every CTA
// computes the prologue redundantly from the producer's vector (<= 32 KB,
// L2-resident), which removes a separate single-CTA kernel and its
// dependency hop from the decode step.
enum GemvPro : int {
  PRO_X8 = 0,         // x8 / xmeta ready in global memory
  PRO_RMSNORM = 1,    // src int16[K]: rmsnorm_fx(src, w, in_f, one_plus) -> DYNQ8
  PRO_DYNQ8 = 2,      // src int16[K]: DYNQ8, in_f given
  PRO_ATTN_GATE = 3,  // src int64[K] (gated attention product): k_a = attn_o_shift,
                      // clip16(rshr(src, k_a)) -> DYNQ8, in_f = QKV_F + GAT_F - k_a
  PRO_ATTN_ACC = 4,   // src int32[K] attention sums acc, src2 int16 q|gate rows of the
                      // q projection: product acc * sigmoid(gate), then as PRO_ATTN_GATE
};

struct GemvPrologue {
  int tag_op1;        // 0: plain input; else the input words are tagged by op tag_op1 - 1
  int mode;
  const void *src;
  const void *src2;   // PRO_ATTN_ACC: q|gate rows ([K/256][512] int16)
  const int32_t *w;   // PRO_RMSNORM gains
  int in_f;
  int one_plus;
  XQ xq_out;          // optional: block 0 stores the computed x8 / meta here
  int *dbg;           // optional: PRO_ATTN_GATE stores k_a here (block 0)
};

struct GemvSeg {
  const uint8_t *w;    // packed image row 0
  const uint8_t *w2;   // paired image (GM_SILU_MUL: up), else null
  void *out;           // output base (indexed by out_row0 + row)
  int64_t *p_out;      // optional int64 p per row (debug / API), nullable
  int rows;            // rows of this segment
  int unit_begin;      // first unit index (units: row pairs, or paired rows)
  int e, e2;           // weight exponents
  int out_f, out_f2;   // output fraction bits (TO16/TO64/RESID/SILU_MUL)
  int mode;
  int out_row0;
  void *aux_out;      // GM_CONV / GM_GATE_*: second output (see GemvMode)
  void *aux0;         // GM_CONV: int16 conv ring [rows][4]; GM_GATE_A: int32 dt_bias (Q12)
  const void *aux1;   // GM_CONV: int32 conv weights [rows][4] (Q.CW_F); GM_GATE_A: int32 A (Q15)
  const int *T;       // GM_CONV: tokens already in the window (ring slot T % 4)
  int tag_op1;        // 0: plain outputs; else tagged words from op tag_op1 - 1 (TO16, RESID,
                      // SILU_MUL: out; CONV, GATE_*: aux_out, and out is skipped when null)
  // optional (GM_RESID): residual statistics of the layer output, the
  // reference's FxRunner.resid_max / resid_clip (ref/fidelity_check.py:
  // 430-431): rstat[0] = max |out| (atomicMax), rstat[1] += the outputs at
  // the int16 rails (out >= 32767 or out <= -32768)
  unsigned long long *rstat;
};

struct GemvArgs {
  GemvSeg seg[GEMV_MAX_SEG];
  int nseg;
  int total_units;
  int K;
  int stride;          // bytes per packed row (ref/w4a8_ref.py:111-114)
  int g;               // group size 128 or 64
  int sh;              // final shift (same for all segments: same K)
  int rows_per_stage;  // set by launch_gemv
  int stages;          // set by launch_gemv
  const int8_t *x8;
  const int *xmeta;    // {e_x, in_f}, nullable (then 0, 0)
  GemvPrologue pro;    // mode PRO_X8 uses x8 / xmeta
  unsigned long long *argmax_key;
  uint32_t *err;
  unsigned *abort_flag;   // persistent kernel: global abort flag polled by bounded tag waits
  // persistent kernel, row-sharded across nrank GPUs: every tagged output
  // word is also stored into each rank's twin buffer, at the local address
  // + peer_delta[r] (CUDA IPC mappings over NVLink; own rank: delta 0)
  int nrank;
  long long peer_delta[F5_MAX_RANKS];
};

cudaError_t launch_gemv(const GemvArgs &a, cudaStream_t st, bool pdl, int max_blocks);

// ---- vector kernels ----
struct NormArgs {
  const int16_t *x16;       // input vector (n = 4096)
  int16_t *x16_store;       // when tok is given: embedding row copied here
  const int16_t *emb;       // embedding table [vocab][n] or null
  const int *tok;           // device token id (with emb), nullable
  const int32_t *w;         // norm weight (Q14, or Q12 pre-folded)
  int n, in_f, one_plus;
  int16_t *xn_out;          // optional normalised vector
  XQ out;                   // DYNQ8 of the normalised vector
};
cudaError_t launch_rmsnorm_dynq8(const NormArgs &a, cudaStream_t st, bool pdl);

struct Dynq8Args {
  const int16_t *x16;
  int n, in_f;
  XQ out;
};
cudaError_t launch_dynq8(const Dynq8Args &a, cudaStream_t st, bool pdl);

// elementwise primitive evaluation (parity tests of the integer law)
enum PrimOp : int {
  PR_RSHR = 0, PR_SIGMOID = 1, PR_SOFTPLUS = 2, PR_SILU = 3, PR_EXP_NEG = 4,
  PR_RSQRT = 5, PR_RECIP = 6, PR_BF_SHIFT = 7, PR_DYNQ8_E = 8,
  PR_DN_NORM_SCALE = 9, PR_EPS_NORM_SCALE = 10, PR_EXP2_FRAC = 11,
};
cudaError_t launch_prim(int op, const int64_t *in, const int64_t *in2, int64_t *out,
                        int64_t *out2, int n, int arg0, int arg1, cudaStream_t st);

}  // namespace f5
