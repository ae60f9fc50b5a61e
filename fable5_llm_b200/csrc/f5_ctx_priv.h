// Private layout of the model context shared by the single-sequence engines
// (f5_ctx.cu) and the batched engine (f5_bctx.cu), which borrows a loaded
// context's weights.
#pragma once
#include <vector>

#include "../../include/f5b200.h"
#include "f5_kernels.cuh"
#include "f5_mega.cuh"

namespace f5 {
// ---------------------------------------------------------------------------
constexpr int H = 4096, FFN = 12288, NQ = 16, NKV = 4, HD = 256, ROT = 64;
constexpr int LNH = 32, LNKH = 16, LDK = 128, LDV = 128;
constexpr int LKD = LNKH * LDK, LVD = LNH * LDV, CONV_DIM = 2 * LKD + LVD;
constexpr int NSLOT = 11;

struct DevMat {
  uint8_t *w = nullptr;
  int N = 0, K = 0, g = 128, e = 0, sh = 0, stride = 0;
  int row0 = 0, rows = 0;   // this rank's rows (split_rows law)
};

struct Layer {
  bool attn = false;
  DevMat m[NSLOT];
  int32_t *ln1 = nullptr, *ln2 = nullptr;
  int32_t *q_norm = nullptr, *k_norm = nullptr;
  int32_t *conv_w = nullptr, *dt_bias = nullptr, *A = nullptr, *norm_w = nullptr;
  // state
  int16_t *conv = nullptr;   // [CONV_DIM][4] ring
  int16_t *S = nullptr;      // [LNH][LDK][LDV]
  int8_t *k8 = nullptr, *ke = nullptr, *v8 = nullptr, *ve = nullptr;
  int *kh = nullptr;         // [LNH] last block-float shifts
  int *ka = nullptr;         // last attention k_a
};

}  // namespace f5

struct f5_ctx {
  f5_config cfg;
  int device = 0;
  cudaStream_t st = nullptr;
  std::vector<f5::Layer> L;
  f5::DevMat head;
  int32_t *ln_f = nullptr;
  int16_t *emb = nullptr;
  int16_t *rope = nullptr;
  int rope_npos = 0;
  // activations
  int16_t *x16 = nullptr, *qkv16 = nullptr, *z16 = nullptr, *b16 = nullptr, *a16 = nullptr;
  int16_t *on16 = nullptr, *qg16 = nullptr, *k16 = nullptr, *v16 = nullptr, *prod16 = nullptr;
  int16_t *qkvc16 = nullptr;   // post-conv q | k | v of a DeltaNet layer
  int32_t *gates = nullptr;    // [2][LNH] beta | decay of a DeltaNet layer
  int64_t *prod64 = nullptr;
  int8_t *x8 = nullptr;
  int *xmeta = nullptr;
  unsigned long long *key = nullptr, *stats = nullptr;
  uint32_t *err = nullptr;
  f5::StepParams *params = nullptr;    // device
  f5::StepParams *h_params = nullptr;  // pinned host mirror
  struct Timed {
    cudaEvent_t a, b;
    int kind;
    double bytes;
  };
  bool timing = false;         // bracket every launch with events (f5_ctx_time_step)
  std::vector<Timed> timed;
  int32_t *logits = nullptr;   // [vocab] y32 of the LM head when enabled
  int32_t *prompt = nullptr;   // [max_T] tokens of f5_decode_prefill
  // TOPK-32 capture (f5_ctx_topk): chunk lists, result, head-prologue operand and {e_x, in_f}
  void *tk_ws = nullptr;
  f5_topk32 *tk_out = nullptr;
  int8_t *tk_xt = nullptr;
  int *tk_xmeta = nullptr;
  bool want_logits = false;
  cudaGraphExec_t step_exec = nullptr;
  bool graph_dirty = true;
  // persistent engine
  int engine = -1;                      // -1 auto (persistent when it fits), else F5_ENGINE_*
  bool mega_dirty = true;
  f5::MegaOp *d_ops = nullptr;          // device op list
  unsigned *d_bars = nullptr;           // barrier counters (+ abort flag, final arrivals)
  uint4 *d_attacc = nullptr;            // per attention layer: score max, exp sum, PV sums
  f5::MegaArgs margs = {};
  int mega_grid = 0;
  size_t mega_smem = 0;
  std::vector<f5::MegaOp> *emit = nullptr;   // enqueue_step in emit mode
  int emit_err = 0;
  int emit_nbar = 0;
  // dataflow-tagged twins (uint32 words) of the activation buffers the
  // persistent program passes between ops, and each twin's last writer op
  struct Twin {
    void *plain;
    size_t plain_bytes, elem;
    uint32_t *tagged;
    int last_op1;
  };
  std::vector<Twin> twins;
  uint32_t *twin_mem = nullptr;
  size_t twin_bytes = 0;        // twins + the cross-rank argmax key slots at the end
  unsigned long long *xkey = nullptr;
  // row sharding: peers' twin allocations mapped through CUDA IPC
  void *peer_base[f5::F5_MAX_RANKS] = {};
  long long peer_delta[f5::F5_MAX_RANKS] = {};
  bool peers_attached = false;
  std::vector<void *> allocs;
};
