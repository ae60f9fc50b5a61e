// Batched decode context: B independent sequences over one loaded model.
//
// The reference decodes one sequence at a time (ref/fidelity_check.py:
// 404-448 FxRunner.step); B sequences are B independent runs of that step.
// Here they share the model context's weights (borrowed, not copied) and
// every projection of the step becomes a W4A8 GEMM on the tensor cores
// (f5_bgemm.cu): the B quantized inputs against one weight image.  Each
// sequence owns its decode state (DeltaNet recurrent states, conv windows,
// KV caches, positions) laid out sequence-major, so the vector stages run
// as the single-sequence kernels with one more grid dimension.
//
// Step program (CUDA graph, programmatic dependent launch between kernels):
//   begin: x16[b] = emb[tok[b]], argmax keys cleared
//   per layer, per projection group: k_bprep (the GEMV prologue of each
//   sequence: RMSNorm / DYNQ8 / attention gate -> x8 tiles), k_bgemm,
//   k_bepi (the GEMV epilogue of each (sequence, row): conv4 + SiLU, gates,
//   residual adds, silu(g) * u); the DeltaNet and attention cores in
//   between, one grid slice per sequence
//   LM head: the GEMM reduces each sequence's argmax; end: next token,
//   advance T / pos per sequence.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/f5b200.h"
#include "f5_attn.cuh"
#include "f5_topk.cuh"
#include "f5_batch.cuh"
#include "f5_capi_util.h"
#include "f5_ctx_priv.h"
#include "f5_dn.cuh"
#include "f5_gemv_core.cuh"
#include "f5_int.cuh"

namespace f5 {

__global__ void k_bstep_begin(StepParams *p, const int16_t *emb, int vocab, int Hd, int16_t *x16,
                              unsigned long long *key) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.x;
  int tok = p[b].tok;
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) atomicOr(&p[b].err, DERR_RANGE);
    tok = 0;
  }
  for (int i = threadIdx.x; i < Hd; i += blockDim.x) x16[(size_t)b * Hd + i] = emb[(size_t)tok * Hd + i];
  if (threadIdx.x == 0) key[b] = 0ull;
}

__global__ void k_bstep_end(StepParams *p, const unsigned long long *key, const uint32_t *err, int B, int advance) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = threadIdx.x;
  if (b >= B) return;
  const unsigned long long k = key[b];
  const int row = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
  const int val = (int)((uint32_t)(k >> 32) ^ 0x80000000u);
  p[b].next_tok = row;
  p[b].max_val = val;
  p[b].err |= *err;
  if (advance) {
    p[b].tok = row;
    p[b].pos += 1;
    p[b].T += 1;
    p[b].steps += 1;
  }
}

// Causal conv4 + SiLU of one prompt chunk's pre-conv projections, token by
// token (ref/layer_fixed.py:1511-1520): channel ch of token t reads the
// ring's three previous inputs, and its own input then replaces the oldest
// slot -- the GM_CONV epilogue of C consecutive decode steps.  One thread
// per channel, the 4-slot ring held in registers across the chunk.
__global__ void k_conv_seq(const int16_t *pre, int16_t *out, int16_t *ring, const int32_t *cw, int C,
                           const StepParams *pp, int nch) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= nch) return;
  const int T0 = pp[0].T;
  uint2 rw = *reinterpret_cast<const uint2 *>(ring + (size_t)ch * 4);
  const int4 w = *reinterpret_cast<const int4 *>(cw + (size_t)ch * 4);
  for (int t = 0; t < C; ++t) {
    const int T = T0 + t;
    const long long v = pre[(size_t)t * nch + ch];
    out[(size_t)t * nch + ch] = (int16_t)conv_silu(v, rw, w, T);
    const uint32_t hv = (uint32_t)(uint16_t)(int16_t)v;
    uint32_t &word = (T & 2) ? rw.y : rw.x;
    word = (T & 1) ? ((word & 0x0000FFFFu) | (hv << 16)) : ((word & 0xFFFF0000u) | hv);
  }
  *reinterpret_cast<uint2 *>(ring + (size_t)ch * 4) = rw;
}

namespace {

struct BLayer {
  int16_t *conv = nullptr, *S = nullptr;
  int8_t *k8 = nullptr, *ke = nullptr, *v8 = nullptr, *ve = nullptr;
  int *kh = nullptr, *ka = nullptr;
};

// one segment of a batched projection group
struct BSeg {
  const DevMat *m = nullptr, *m2 = nullptr;   // m2: the up image of a gate/up pair
  int mode = GM_TO16, out_f = 0, out_f2 = 0;
  void *out = nullptr;
  long long out_bs = 0;                        // bytes between sequences
  void *aux_out = nullptr;
  long long aux_bs = 0;
  void *aux0 = nullptr;
  long long ring_bs = 0;
  const void *aux1 = nullptr;
};

constexpr size_t PARAM_INTS = sizeof(StepParams) / sizeof(int);

struct BDevGuard {
  int prev = 0;
  explicit BDevGuard(int d) { cudaGetDevice(&prev); cudaSetDevice(d); }
  ~BDevGuard() { cudaSetDevice(prev); }
};

}  // namespace
}  // namespace f5

using namespace f5;

struct f5_bctx {
  f5_ctx *m = nullptr;
  int B = 0, Bp = 0, max_T = 0, device = 0;
  cudaStream_t st = nullptr;
  std::vector<BLayer> L;
  int16_t *x16 = nullptr, *qkv16 = nullptr, *qkvc16 = nullptr, *z16 = nullptr, *b16 = nullptr, *a16 = nullptr;
  int16_t *on16 = nullptr, *qg16 = nullptr, *k16 = nullptr, *v16 = nullptr, *prod16 = nullptr;
  int32_t *gates = nullptr;
  int64_t *prod64 = nullptr;
  int8_t *xt = nullptr;
  int *xmeta = nullptr;
  int64_t *p = nullptr;
  size_t p_words = 0;
  unsigned long long *key = nullptr, *stats = nullptr;
  uint32_t *err = nullptr;
  int32_t *logits = nullptr;   // [B][vocab] y32 of the LM head when enabled (f5_bctx_set_logits)
  bool want_logits = false;
  void *tk_ws = nullptr;       // f5_bctx_topk: chunk lists of B logit rows, B results
  f5_topk32 *tk_out = nullptr;
  StepParams *params = nullptr, *h_params = nullptr;
  StepParams *pparams = nullptr;   // f5_bctx_prefill: one entry per token of the chunk (T, pos, tok)
  int ncol = 0;                    // GEMM columns of the next ops (0: B); prefill chunks set it
  cudaGraphExec_t exec = nullptr;
  bool dirty = true;
  bool pdl = true;             // programmatic dependent launch between the step's kernels
  struct Timed {
    cudaEvent_t a, b;
    int kind;
    double bytes;
  };
  bool timing = false;         // bracket every launch with events (f5_bctx_time_step)
  std::vector<Timed> timed;
  bool sizing = false;         // enqueue walk that only sizes the p scratch
  size_t need_p = 0;
  std::vector<void *> allocs;
};

#define F5_CU(x, what)                        \
  do {                                        \
    int _rc = cuda_status((x), (what));       \
    if (_rc) return _rc;                      \
  } while (0)

namespace f5 {
namespace {

int balloc(f5_bctx *c, void **p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaMalloc");
  c->allocs.push_back(*p);
  return cuda_status(cudaMemsetAsync(*p, 0, bytes, c->st), "cudaMemset");
}
#define F5_BALLOC(c, p, bytes)                                            \
  do {                                                                    \
    int _rc = balloc((c), reinterpret_cast<void **>(&(p)), (bytes));      \
    if (_rc) return _rc;                                                  \
  } while (0)

enum { BK_PREP = 0, BK_GEMM = 1, BK_EPI = 2, BK_DN = 3, BK_ATTN = 4, BK_OTHER = 5, BK_N = 6 };
void tb(f5_bctx *c) {
  if (!c->timing) return;
  f5_bctx::Timed t = {};
  cudaEventCreate(&t.a);
  cudaEventCreate(&t.b);
  cudaEventRecord(t.a, c->st);
  c->timed.push_back(t);
}
void te(f5_bctx *c, int kind, double bytes) {
  if (!c->timing) return;
  f5_bctx::Timed &t = c->timed.back();
  t.kind = kind;
  t.bytes = bytes;
  cudaEventRecord(t.b, c->st);
}

// One batched projection group: prologue -> GEMM -> per-sequence epilogue.
cudaError_t bop(f5_bctx *c, const BSeg *sg, int nseg, int K, const GemvPrologue &pro, long long src_bs,
                long long src2_bs, bool head) {
  const int NG = K / 128;
  BgemmArgs ga = {};
  BepiArgs ea = {};
  int tiles = 0, prow = 0, units = 0, gs = 0;
  for (int i = 0; i < nseg; ++i) {
    const BSeg &s = sg[i];
    const DevMat *ms[2] = {s.m, s.m2};
    const int nm = s.mode == GM_SILU_MUL ? 2 : 1;
    const int p0 = prow;
    for (int k = 0; k < nm; ++k) {
      if (gs >= BG_MAX_SEG) return cudaErrorInvalidValue;
      BgemmSeg &g = ga.seg[gs++];
      g.w = ms[k]->w;
      g.rows = ms[k]->N;
      g.tile_begin = tiles;
      g.p_row0 = prow;
      g.argmax = head ? 1 : 0;
      tiles += (ms[k]->N + BG_TILE - 1) / BG_TILE;
      if (!head) prow += ms[k]->N;
    }
    GemvSeg &e = ea.g.seg[i];
    e.out = s.out;
    e.rows = s.m->N;
    e.unit_begin = units;
    e.e = s.m->e;
    e.e2 = s.m2 ? s.m2->e : 0;
    e.out_f = s.out_f;
    e.out_f2 = s.out_f2;
    e.mode = s.mode;
    e.aux_out = s.aux_out;
    e.aux0 = s.aux0;
    e.aux1 = s.aux1;
    BepiSeg &b = ea.bs[i];
    b.p_row0 = p0;
    b.p_row0_up = p0 + s.m->N;
    b.out_bs = s.out_bs;
    b.aux_bs = s.aux_bs;
    b.ring_bs = s.ring_bs;
    units += s.m->N;
  }
  ga.nseg = gs;
  ga.ntiles = tiles;
  ga.K = K;
  ga.NG = NG;
  ga.stride = sg[0].m->stride;
  ga.sh = sg[0].m->sh;
  ga.S = bgemm_splits(tiles, NG, sm_count(), head);
  const int ncol = c->ncol > 0 ? c->ncol : c->B;
  ga.B = ncol;
  ga.Bp = c->Bp;
  ga.xt = c->xt;
  ga.p = c->p;
  ga.ptot = prow;
  ga.key = head ? c->key : nullptr;
  if (head && c->want_logits) {
    ga.y_out = c->logits;
    ga.y_bs = c->m->cfg.vocab;
  }
  ga.err = c->err;
  if (c->sizing) {
    c->need_p = std::max(c->need_p, (size_t)ga.S * c->Bp * (size_t)prow);
    return cudaSuccess;
  }
  BprepArgs pa = {};
  pa.pro = pro;
  pa.src_bs = src_bs;
  pa.src2_bs = src2_bs;
  pa.K = K;
  pa.NG = NG;
  pa.B = ncol;
  pa.Bp = c->Bp;
  pa.xmeta = c->xmeta;
  pa.xt = c->xt;
  pa.err = c->err;
  cudaError_t e;
  double wbytes = 0;
  for (int i = 0; i < gs; ++i) wbytes += (double)ga.seg[i].rows * ga.stride;
  tb(c);
  e = launch_bprep(pa, c->st, c->pdl);
  te(c, BK_PREP, 0);
  if (e) return e;
  tb(c);
  e = launch_bgemm(ga, c->st, c->pdl, sm_count());
  te(c, BK_GEMM, wbytes);
  if (e) return e;
  if (head) return cudaSuccess;
  ea.g.nseg = nseg;
  ea.g.total_units = units;
  ea.g.K = K;
  ea.g.sh = ga.sh;
  ea.g.err = c->err;
  ea.S = ga.S;
  ea.B = ncol;
  ea.Bp = c->Bp;
  ea.ptot = prow;
  ea.p = c->p;
  ea.xmeta = c->xmeta;
  ea.params = c->params;
  tb(c);
  e = launch_bepi(ea, c->st, c->pdl);
  te(c, BK_EPI, 0);
  return e;
}

cudaError_t enqueue_blayer(f5_bctx *c, int li) {
  const Layer &l = c->m->L[li];
  BLayer &s = c->L[li];
  cudaError_t e;
  GemvPrologue pro = {};
  pro.mode = PRO_RMSNORM;
  pro.src = c->x16;
  pro.w = l.ln1;
  pro.in_f = RS_F;
  pro.one_plus = 1;
  const long long xbs = (long long)H * 2;
  if (!l.attn) {
    // in-projection with conv4 + SiLU and the two gates (ref/layer_fixed.py:1503-1538)
    BSeg sg[4];
    sg[0].m = &l.m[0]; sg[0].mode = GM_CONV; sg[0].out_f = RS_F;
    sg[0].out = c->qkv16; sg[0].out_bs = (long long)CONV_DIM * 2;
    sg[0].aux_out = c->qkvc16; sg[0].aux_bs = (long long)CONV_DIM * 2;
    sg[0].aux0 = s.conv; sg[0].ring_bs = (long long)CONV_DIM * 4 * 2; sg[0].aux1 = l.conv_w;
    sg[1].m = &l.m[1]; sg[1].mode = GM_TO16; sg[1].out_f = QKV_F; sg[1].out = c->z16; sg[1].out_bs = (long long)LVD * 2;
    sg[2].m = &l.m[2]; sg[2].mode = GM_GATE_B; sg[2].out_f = 12; sg[2].out = c->b16; sg[2].out_bs = (long long)LNH * 2;
    sg[2].aux_out = c->gates; sg[2].aux_bs = (long long)2 * LNH * 4;
    sg[3].m = &l.m[3]; sg[3].mode = GM_GATE_A; sg[3].out_f = 12; sg[3].out = c->a16; sg[3].out_bs = (long long)LNH * 2;
    sg[3].aux_out = c->gates + LNH; sg[3].aux_bs = (long long)2 * LNH * 4;
    sg[3].aux0 = l.dt_bias; sg[3].aux1 = l.A;
    if ((e = bop(c, sg, 4, H, pro, xbs, 0, false))) return e;
    if (!c->sizing) {
      DnArgs d = {};
      d.qkvc = c->qkvc16; d.beta = c->gates; d.decay = c->gates + LNH; d.z16 = c->z16; d.norm_w = l.norm_w;
      d.S = s.S; d.on16 = c->on16; d.kh_out = s.kh; d.stats = c->stats; d.err = c->err;
      d.lkd = LKD; d.vrep = LNH / LNKH; d.norm_mode = c->m->cfg.norm_mode;
      DnBatch bs;
      bs.qkvc = CONV_DIM; bs.gates = 2 * LNH; bs.z = LVD; bs.S = (long long)LNH * LDK * LDV; bs.on = LVD; bs.kh = LNH;
      tb(c);
      e = launch_dn_step_b(d, bs, LNH, c->B, c->st, c->pdl);
      te(c, BK_DN, 0);
      if (e) return e;
    }
    GemvPrologue p2 = {};
    p2.mode = PRO_DYNQ8;
    p2.src = c->on16;
    p2.in_f = DN_NORM_F;
    BSeg so;
    so.m = &l.m[4]; so.mode = GM_RESID; so.out_f = RS_F; so.out = c->x16; so.out_bs = xbs;
    if ((e = bop(c, &so, 1, LVD, p2, (long long)LVD * 2, 0, false))) return e;
  } else {
    BSeg sg[3];
    sg[0].m = &l.m[0]; sg[0].out = c->qg16; sg[0].out_bs = (long long)NQ * HD * 2 * 2;
    sg[1].m = &l.m[1]; sg[1].out = c->k16; sg[1].out_bs = (long long)NKV * HD * 2;
    sg[2].m = &l.m[2]; sg[2].out = c->v16; sg[2].out_bs = (long long)NKV * HD * 2;
    for (BSeg &x : sg) { x.mode = GM_TO16; x.out_f = QKV_F; }
    if ((e = bop(c, sg, 3, H, pro, xbs, 0, false))) return e;
    if (!c->sizing) {
      AttnArgs at = {};
      at.qg16 = c->qg16; at.k16 = c->k16; at.v16 = c->v16; at.q_norm = l.q_norm; at.k_norm = l.k_norm;
      at.rope = c->m->rope; at.k8 = s.k8; at.ke = s.ke; at.v8 = s.v8; at.ve = s.ve; at.prod = c->prod64;
      at.T = &c->params->T; at.pos = &c->params->pos; at.err = c->err;
      at.max_T = c->max_T; at.max_pos = c->m->rope_npos; at.nq = NQ; at.nkv = NKV; at.rot = ROT;
      AttnBatch bs;
      bs.qg = (long long)NQ * HD * 2; bs.kv16 = (long long)NKV * HD;
      bs.cache = (long long)NKV * c->max_T * HD; bs.cache_e = (long long)NKV * c->max_T;
      bs.prod = (long long)NQ * HD; bs.params = (long long)PARAM_INTS;
      tb(c);
      e = launch_attn_b(at, bs, c->B, c->st, c->pdl);
      te(c, BK_ATTN, 0);
      if (e) return e;
    }
    GemvPrologue p2 = {};
    p2.mode = PRO_ATTN_GATE;
    p2.src = c->prod64;
    p2.dbg = s.ka;
    BSeg so;
    so.m = &l.m[3]; so.mode = GM_RESID; so.out_f = RS_F; so.out = c->x16; so.out_bs = xbs;
    if ((e = bop(c, &so, 1, NQ * HD, p2, (long long)NQ * HD * 8, 0, false))) return e;
  }
  // MLP (ref/layer_fixed.py:1597-1604)
  GemvPrologue p3 = {};
  p3.mode = PRO_RMSNORM;
  p3.src = c->x16;
  p3.w = l.ln2;
  p3.in_f = RS_F;
  p3.one_plus = 1;
  BSeg gu;
  gu.m = &l.m[8]; gu.m2 = &l.m[9]; gu.mode = GM_SILU_MUL; gu.out_f = 12; gu.out_f2 = RS_F;
  gu.out = c->prod16; gu.out_bs = (long long)FFN * 2;
  if ((e = bop(c, &gu, 1, H, p3, xbs, 0, false))) return e;
  GemvPrologue p4 = {};
  p4.mode = PRO_DYNQ8;
  p4.src = c->prod16;
  p4.in_f = RS_F;
  BSeg sd;
  sd.m = &l.m[10]; sd.mode = GM_RESID; sd.out_f = RS_F; sd.out = c->x16; sd.out_bs = xbs;
  return bop(c, &sd, 1, FFN, p4, (long long)FFN * 2, 0, false);
}

cudaError_t launch_pdl_b(const void *fn, void **args, dim3 grid, dim3 block, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t enqueue_bstep(f5_bctx *c) {
  cudaError_t e;
  if (!c->sizing) {
    StepParams *p = c->params;
    const int16_t *emb = c->m->emb;
    int vocab = c->m->cfg.vocab, hd = H;
    int16_t *x = c->x16;
    unsigned long long *k = c->key;
    void *args[] = {&p, &emb, &vocab, &hd, &x, &k};
    if ((e = launch_pdl_b((const void *)k_bstep_begin, args, dim3(c->B), dim3(256), c->st, c->pdl))) return e;
  }
  for (int li = 0; li < (int)c->L.size(); ++li)
    if ((e = enqueue_blayer(c, li))) return e;
  GemvPrologue pf = {};
  pf.mode = PRO_RMSNORM;
  pf.src = c->x16;
  pf.w = c->m->ln_f;
  pf.in_f = RS_F;
  pf.one_plus = 0;   // ln_f pre-folded (1+w) at Q3.12
  BSeg sh;
  sh.m = &c->m->head;
  sh.mode = GM_ARGMAX;
  if ((e = bop(c, &sh, 1, H, pf, (long long)H * 2, 0, true))) return e;
  if (!c->sizing) {
    StepParams *p = c->params;
    const unsigned long long *k = c->key;
    const uint32_t *er = c->err;
    int B = c->B, adv = 1;
    void *args[] = {&p, &k, &er, &B, &adv};
    if ((e = launch_pdl_b((const void *)k_bstep_end, args, dim3(1), dim3(64), c->st, c->pdl))) return e;
  }
  return cudaSuccess;
}

int build_bgraph(f5_bctx *c) {
  if (!c->dirty && c->exec) return F5_OK;
  if (c->exec) {
    cudaGraphExecDestroy(c->exec);
    c->exec = nullptr;
  }
  cudaGraph_t g = nullptr;
  F5_CU(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal), "capture");
  cudaError_t e = enqueue_bstep(c);
  cudaError_t e2 = cudaStreamEndCapture(c->st, &g);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return cuda_status(e != cudaSuccess ? e : e2, "batched step capture");
  }
  e = cudaGraphInstantiate(&c->exec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return cuda_status(e, "batched graph instantiate");
  c->dirty = false;
  return F5_OK;
}

int bfinish(f5_bctx *c, const char *what) {
  cudaError_t e = cudaStreamSynchronize(c->st);
  if (e != cudaSuccess) return cuda_status(e, what);
  F5_CU(cudaMemcpy(c->h_params, c->params, sizeof(StepParams) * c->B, cudaMemcpyDeviceToHost), what);
  uint32_t any = 0;
  for (int b = 0; b < c->B; ++b) any |= c->h_params[b].err;
  if (any & DERR_TIMEOUT) return set_error(F5_ETIMEOUT, "%s: a bounded device wait expired", what);
  if (any & DERR_Y32_OVERFLOW) return set_error(F5_EOVERFLOW, "%s: |y32| >= 2^31", what);
  if (any & DERR_KV_FULL) return set_error(F5_ESTATE, "%s: KV cache full (max_T)", what);
  if (any & DERR_RANGE) return set_error(F5_EINVAL, "%s: input out of range", what);
  return F5_OK;
}

// device buffer of (what, layer) for sequence seq, with its per-sequence bytes
int bbuf(f5_bctx *c, int what, int layer, int seq, uint8_t **ptr, size_t *bytes) {
  if (seq < 0 || seq >= c->B) return set_error(F5_EINVAL, "sequence %d outside [0, %d)", seq, c->B);
  const bool per_layer = what == F5_BUF_DN_S || what == F5_BUF_DN_CONV || what == F5_BUF_DN_KH ||
                         what == F5_BUF_K8 || what == F5_BUF_KE || what == F5_BUF_V8 || what == F5_BUF_VE ||
                         what == F5_BUF_KA;
  if (per_layer && (layer < 0 || layer >= (int)c->L.size())) return set_error(F5_EINVAL, "layer %d", layer);
  const bool attn = per_layer && c->m->L[layer].attn;
  const size_t T = (size_t)c->max_T;
  uint8_t *base = nullptr;
  size_t n = 0;
  switch (what) {
    case F5_BUF_X16: base = (uint8_t *)c->x16; n = (size_t)H * 2; break;
    case F5_BUF_QKV16: base = (uint8_t *)c->qkv16; n = (size_t)CONV_DIM * 2; break;
    case F5_BUF_Z16: base = (uint8_t *)c->z16; n = (size_t)LVD * 2; break;
    case F5_BUF_B16: base = (uint8_t *)c->b16; n = (size_t)LNH * 2; break;
    case F5_BUF_A16: base = (uint8_t *)c->a16; n = (size_t)LNH * 2; break;
    case F5_BUF_K16: base = (uint8_t *)c->k16; n = (size_t)NKV * HD * 2; break;
    case F5_BUF_V16: base = (uint8_t *)c->v16; n = (size_t)NKV * HD * 2; break;
    case F5_BUF_PROD64: base = (uint8_t *)c->prod64; n = (size_t)NQ * HD * 8; break;
    case F5_BUF_QKVC16: base = (uint8_t *)c->qkvc16; n = (size_t)CONV_DIM * 2; break;
    case F5_BUF_GATES: base = (uint8_t *)c->gates; n = (size_t)2 * LNH * 4; break;
    case F5_BUF_LOGITS: if (!c->logits) break; base = (uint8_t *)c->logits; n = (size_t)c->m->cfg.vocab * 4; break;
    case F5_BUF_ON16: base = (uint8_t *)c->on16; n = (size_t)LVD * 2; break;
    case F5_BUF_QG16: base = (uint8_t *)c->qg16; n = (size_t)NQ * HD * 4; break;
    case F5_BUF_PROD16: base = (uint8_t *)c->prod16; n = (size_t)FFN * 2; break;
    case F5_BUF_DN_S: if (attn) break; base = (uint8_t *)c->L[layer].S; n = (size_t)LNH * LDK * LDV * 2; break;
    case F5_BUF_DN_CONV: if (attn) break; base = (uint8_t *)c->L[layer].conv; n = (size_t)CONV_DIM * 4 * 2; break;
    case F5_BUF_DN_KH: if (attn) break; base = (uint8_t *)c->L[layer].kh; n = (size_t)LNH * 4; break;
    case F5_BUF_K8: if (!attn) break; base = (uint8_t *)c->L[layer].k8; n = NKV * T * HD; break;
    case F5_BUF_V8: if (!attn) break; base = (uint8_t *)c->L[layer].v8; n = NKV * T * HD; break;
    case F5_BUF_KE: if (!attn) break; base = (uint8_t *)c->L[layer].ke; n = NKV * T; break;
    case F5_BUF_VE: if (!attn) break; base = (uint8_t *)c->L[layer].ve; n = NKV * T; break;
    case F5_BUF_KA: if (!attn) break; base = (uint8_t *)c->L[layer].ka; n = 4; break;
    default: break;
  }
  if (!base) return set_error(F5_EINVAL, "buffer %d is not held by layer %d of a batched context", what, layer);
  *ptr = base + (size_t)seq * n;
  *bytes = n;
  return F5_OK;
}

// One chunk of layer-major prompt ingestion for sequence `seq`: the C
// tokens in pparams[0..C) (tok, T = T0 + t, pos = pos0 + t) are the C
// columns of every projection GEMM, while the conv window, the DeltaNet
// recurrence and the KV appends -- the parts that carry state from one token
// to the next -- run token by token in order.  Every value therefore equals
// what C sequential decode steps of that sequence compute.  `last`: the LM
// head runs too and pparams[t].next_tok receives each column's argmax.
cudaError_t enqueue_prefill_chunk(f5_bctx *c, int seq, int C, bool last) {
  cudaError_t e;
  c->ncol = C;
  {
    StepParams *p = c->pparams;
    const int16_t *emb = c->m->emb;
    int vocab = c->m->cfg.vocab, hd = H;
    int16_t *x = c->x16;
    unsigned long long *k = c->key;
    void *args[] = {&p, &emb, &vocab, &hd, &x, &k};
    if ((e = launch_pdl_b((const void *)k_bstep_begin, args, dim3(C), dim3(256), c->st, c->pdl))) return e;
  }
  const long long xbs = (long long)H * 2;
  for (int li = 0; li < (int)c->L.size(); ++li) {
    const Layer &l = c->m->L[li];
    BLayer &s = c->L[li];
    GemvPrologue pro = {};
    pro.mode = PRO_RMSNORM;
    pro.src = c->x16;
    pro.w = l.ln1;
    pro.in_f = RS_F;
    pro.one_plus = 1;
    if (!l.attn) {
      BSeg sg[4];
      sg[0].m = &l.m[0]; sg[0].mode = GM_TO16; sg[0].out_f = RS_F;     // pre-conv inputs, convolved below
      sg[0].out = c->qkv16; sg[0].out_bs = (long long)CONV_DIM * 2;
      sg[1].m = &l.m[1]; sg[1].mode = GM_TO16; sg[1].out_f = QKV_F; sg[1].out = c->z16; sg[1].out_bs = (long long)LVD * 2;
      sg[2].m = &l.m[2]; sg[2].mode = GM_GATE_B; sg[2].out_f = 12; sg[2].out = c->b16; sg[2].out_bs = (long long)LNH * 2;
      sg[2].aux_out = c->gates; sg[2].aux_bs = (long long)2 * LNH * 4;
      sg[3].m = &l.m[3]; sg[3].mode = GM_GATE_A; sg[3].out_f = 12; sg[3].out = c->a16; sg[3].out_bs = (long long)LNH * 2;
      sg[3].aux_out = c->gates + LNH; sg[3].aux_bs = (long long)2 * LNH * 4;
      sg[3].aux0 = l.dt_bias; sg[3].aux1 = l.A;
      if ((e = bop(c, sg, 4, H, pro, xbs, 0, false))) return e;
      {
        const int16_t *pre = c->qkv16;
        int16_t *out = c->qkvc16;
        int16_t *ring = s.conv + (size_t)seq * CONV_DIM * 4;
        const int32_t *cw = l.conv_w;
        int Cc = C, nch = CONV_DIM;
        const StepParams *pp = c->pparams;
        void *args[] = {&pre, &out, &ring, &cw, &Cc, &pp, &nch};
        if ((e = launch_pdl_b((const void *)k_conv_seq, args, dim3(CONV_DIM / 256), dim3(256), c->st, c->pdl)))
          return e;
      }
      DnBatch bs;
      bs.qkvc = CONV_DIM; bs.gates = 2 * LNH; bs.z = LVD; bs.S = (long long)LNH * LDK * LDV; bs.on = LVD; bs.kh = LNH;
      {
        DnArgs d = {};
        d.qkvc = c->qkvc16;
        d.beta = c->gates;
        d.decay = c->gates + LNH;
        d.z16 = c->z16;
        d.norm_w = l.norm_w;
        d.S = s.S + (size_t)seq * LNH * LDK * LDV;
        d.on16 = c->on16;
        d.kh_out = s.kh + (size_t)seq * LNH;
        d.stats = c->stats;
        d.err = c->err;
        d.lkd = LKD; d.vrep = LNH / LNKH; d.norm_mode = c->m->cfg.norm_mode;
        // all C tokens in one launch, the state kept in shared memory
        // between them (no programmatic early launch: the state is read
        // right after the previous kernels)
        if ((e = launch_dn_scan(d, bs, LNH, C, c->st))) return e;
      }
      GemvPrologue p2 = {};
      p2.mode = PRO_DYNQ8;
      p2.src = c->on16;
      p2.in_f = DN_NORM_F;
      BSeg so;
      so.m = &l.m[4]; so.mode = GM_RESID; so.out_f = RS_F; so.out = c->x16; so.out_bs = xbs;
      if ((e = bop(c, &so, 1, LVD, p2, (long long)LVD * 2, 0, false))) return e;
    } else {
      BSeg sg[3];
      sg[0].m = &l.m[0]; sg[0].out = c->qg16; sg[0].out_bs = (long long)NQ * HD * 2 * 2;
      sg[1].m = &l.m[1]; sg[1].out = c->k16; sg[1].out_bs = (long long)NKV * HD * 2;
      sg[2].m = &l.m[2]; sg[2].out = c->v16; sg[2].out_bs = (long long)NKV * HD * 2;
      for (BSeg &x : sg) { x.mode = GM_TO16; x.out_f = QKV_F; }
      if ((e = bop(c, sg, 3, H, pro, xbs, 0, false))) return e;
      AttnBatch bs;
      bs.qg = (long long)NQ * HD * 2; bs.kv16 = (long long)NKV * HD;
      bs.cache = (long long)NKV * c->max_T * HD; bs.cache_e = (long long)NKV * c->max_T;
      bs.prod = (long long)NQ * HD; bs.params = (long long)PARAM_INTS;
      const size_t cs = (size_t)seq * NKV * c->max_T;
      for (int t = 0; t < C; ++t) {
        AttnArgs at = {};
        at.qg16 = c->qg16 + (size_t)t * NQ * HD * 2;
        at.k16 = c->k16 + (size_t)t * NKV * HD;
        at.v16 = c->v16 + (size_t)t * NKV * HD;
        at.q_norm = l.q_norm; at.k_norm = l.k_norm; at.rope = c->m->rope;
        at.k8 = s.k8 + cs * HD; at.ke = s.ke + cs; at.v8 = s.v8 + cs * HD; at.ve = s.ve + cs;
        at.prod = c->prod64 + (size_t)t * NQ * HD;
        at.T = &c->pparams[t].T; at.pos = &c->pparams[t].pos; at.err = c->err;
        at.max_T = c->max_T; at.max_pos = c->m->rope_npos; at.nq = NQ; at.nkv = NKV; at.rot = ROT;
        // no programmatic early launch: the kernel copies its cached K rows
        // before its dependency wait, and the previous token appended one
        if ((e = launch_attn_b(at, bs, 1, c->st, false))) return e;
      }
      GemvPrologue p2 = {};
      p2.mode = PRO_ATTN_GATE;
      p2.src = c->prod64;
      BSeg so;
      so.m = &l.m[3]; so.mode = GM_RESID; so.out_f = RS_F; so.out = c->x16; so.out_bs = xbs;
      if ((e = bop(c, &so, 1, NQ * HD, p2, (long long)NQ * HD * 8, 0, false))) return e;
    }
    GemvPrologue p3 = {};
    p3.mode = PRO_RMSNORM;
    p3.src = c->x16;
    p3.w = l.ln2;
    p3.in_f = RS_F;
    p3.one_plus = 1;
    BSeg gu;
    gu.m = &l.m[8]; gu.m2 = &l.m[9]; gu.mode = GM_SILU_MUL; gu.out_f = 12; gu.out_f2 = RS_F;
    gu.out = c->prod16; gu.out_bs = (long long)FFN * 2;
    if ((e = bop(c, &gu, 1, H, p3, xbs, 0, false))) return e;
    GemvPrologue p4 = {};
    p4.mode = PRO_DYNQ8;
    p4.src = c->prod16;
    p4.in_f = RS_F;
    BSeg sd;
    sd.m = &l.m[10]; sd.mode = GM_RESID; sd.out_f = RS_F; sd.out = c->x16; sd.out_bs = xbs;
    if ((e = bop(c, &sd, 1, FFN, p4, (long long)FFN * 2, 0, false))) return e;
  }
  if (last) {
    GemvPrologue pf = {};
    pf.mode = PRO_RMSNORM;
    pf.src = c->x16;
    pf.w = c->m->ln_f;
    pf.in_f = RS_F;
    pf.one_plus = 0;
    BSeg sh;
    sh.m = &c->m->head;
    sh.mode = GM_ARGMAX;
    if ((e = bop(c, &sh, 1, H, pf, (long long)H * 2, 0, true))) return e;
    StepParams *p = c->pparams;
    const unsigned long long *k = c->key;
    const uint32_t *er = c->err;
    int B = C, adv = 0;
    void *args[] = {&p, &k, &er, &B, &adv};
    if ((e = launch_pdl_b((const void *)k_bstep_end, args, dim3(1), dim3(64), c->st, c->pdl))) return e;
  }
  c->ncol = 0;
  return cudaSuccess;
}

}  // namespace
}  // namespace f5

extern "C" {

int f5_bctx_create(f5_ctx *m, int batch, int max_T, f5_bctx **out) {
  if (!m || !out) return set_error(F5_EINVAL, "f5_bctx_create: null argument");
  *out = nullptr;
  if (batch < 1 || batch > 64) return set_error(F5_EINVAL, "f5_bctx_create: batch %d outside [1, 64]", batch);
  if (max_T < 16 || max_T % 16) return set_error(F5_EINVAL, "f5_bctx_create: max_T must be a positive multiple of 16");
  if (m->cfg.world_size != 1) return set_error(F5_EINVAL, "f5_bctx_create: the model context must hold every row (world_size 1)");
  for (size_t i = 0; i < m->L.size(); ++i)
    for (int s = 0; s < NSLOT; ++s) {
      const bool used = (s >= 8 && s <= 10) || (m->L[i].attn ? s <= 3 : s <= 4);
      if (used && !m->L[i].m[s].w) return set_error(F5_ESTATE, "f5_bctx_create: layer %zu slot %d not uploaded", i, s);
      if (used && m->L[i].m[s].g != 128) return set_error(F5_EINVAL, "f5_bctx_create: g=128 images only");
    }
  if (!m->head.w || !m->emb || !m->rope || !m->ln_f) return set_error(F5_ESTATE, "f5_bctx_create: model not fully loaded");
  f5_bctx *c = new f5_bctx();
  c->m = m;
  c->B = batch;
  c->Bp = batch <= 16 ? 16 : (batch <= 32 ? 32 : 64);
  c->max_T = max_T;
  c->device = m->device;
  if (const char *v = getenv("F5_BATCH_PDL")) c->pdl = atoi(v) != 0;
  BDevGuard dg(c->device);
  int rc = F5_OK;
  auto fail = [&](int r) { f5_bctx_destroy(c); return r; };
  if (cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking) != cudaSuccess)
    return fail(set_error(F5_ECUDA, "stream"));
  const size_t B = batch;
#define BA(p, n) do { if ((rc = balloc(c, reinterpret_cast<void **>(&(p)), (n)))) return fail(rc); } while (0)
  c->L.resize(m->L.size());
  for (size_t i = 0; i < m->L.size(); ++i) {
    BLayer &s = c->L[i];
    if (!m->L[i].attn) {
      BA(s.conv, B * CONV_DIM * 4 * 2);
      BA(s.S, B * LNH * LDK * LDV * 2);
      BA(s.kh, B * LNH * 4);
    } else {
      BA(s.k8, B * NKV * max_T * HD);
      BA(s.v8, B * NKV * max_T * HD);
      BA(s.ke, B * NKV * max_T);
      BA(s.ve, B * NKV * max_T);
      BA(s.ka, B * 4);
    }
  }
  BA(c->x16, B * H * 2);
  BA(c->qkv16, B * CONV_DIM * 2);
  BA(c->qkvc16, B * CONV_DIM * 2);
  BA(c->z16, B * LVD * 2);
  BA(c->b16, B * LNH * 2);
  BA(c->a16, B * LNH * 2);
  BA(c->gates, B * 2 * LNH * 4);
  BA(c->on16, B * LVD * 2);
  BA(c->qg16, B * NQ * HD * 2 * 2);
  BA(c->k16, B * NKV * HD * 2);
  BA(c->v16, B * NKV * HD * 2);
  BA(c->prod16, B * FFN * 2);
  BA(c->prod64, B * NQ * HD * 8);
  BA(c->xt, (size_t)(FFN / 128) * c->Bp * 128);   // rows >= B stay zero
  BA(c->xmeta, (size_t)c->Bp * 2 * 4);
  BA(c->key, (size_t)c->Bp * 8);
  BA(c->stats, 8);
  BA(c->err, 4);
  BA(c->params, B * sizeof(StepParams));
  BA(c->pparams, B * sizeof(StepParams));
  if (cudaMallocHost(&c->h_params, B * sizeof(StepParams)) != cudaSuccess)
    return fail(set_error(F5_ENOMEM, "pinned params"));
  memset(c->h_params, 0, B * sizeof(StepParams));
  // size the partial-p scratch with a dry walk of the step
  c->sizing = true;
  enqueue_bstep(c);
  c->sizing = false;
  BA(c->p, std::max<size_t>(c->need_p, 1) * 8);
#undef BA
  if ((rc = cuda_status(cudaStreamSynchronize(c->st), "f5_bctx_create"))) return fail(rc);
  *out = c;
  return F5_OK;
}

int f5_bctx_destroy(f5_bctx *c) {
  if (!c) return F5_OK;
  BDevGuard dg(c->device);
  if (c->st) cudaStreamSynchronize(c->st);
  if (c->exec) cudaGraphExecDestroy(c->exec);
  for (void *p : c->allocs) cudaFree(p);
  if (c->h_params) cudaFreeHost(c->h_params);
  if (c->st) cudaStreamDestroy(c->st);
  delete c;
  return F5_OK;
}

int f5_bctx_reset(f5_bctx *c) {
  if (!c) return set_error(F5_EINVAL, "null batched context");
  BDevGuard dg(c->device);
  for (BLayer &s : c->L) {
    const size_t B = c->B;
    if (s.S) {
      F5_CU(cudaMemsetAsync(s.S, 0, B * LNH * LDK * LDV * 2, c->st), "reset");
      F5_CU(cudaMemsetAsync(s.conv, 0, B * CONV_DIM * 4 * 2, c->st), "reset");
      F5_CU(cudaMemsetAsync(s.kh, 0, B * LNH * 4, c->st), "reset");
    } else {
      F5_CU(cudaMemsetAsync(s.k8, 0, B * NKV * c->max_T * HD, c->st), "reset");
      F5_CU(cudaMemsetAsync(s.v8, 0, B * NKV * c->max_T * HD, c->st), "reset");
      F5_CU(cudaMemsetAsync(s.ke, 0, B * NKV * c->max_T, c->st), "reset");
      F5_CU(cudaMemsetAsync(s.ve, 0, B * NKV * c->max_T, c->st), "reset");
    }
  }
  F5_CU(cudaMemsetAsync(c->stats, 0, 8, c->st), "reset");
  F5_CU(cudaMemsetAsync(c->err, 0, 4, c->st), "reset");
  F5_CU(cudaMemsetAsync(c->params, 0, sizeof(StepParams) * c->B, c->st), "reset");
  return cuda_status(cudaStreamSynchronize(c->st), "f5_bctx_reset");
}

int f5_bctx_set_position(f5_bctx *c, int seq, int T, int pos) {
  if (!c) return set_error(F5_EINVAL, "null batched context");
  if (T < 0 || T > c->max_T || pos < 0) return set_error(F5_EINVAL, "set_position: T=%d pos=%d", T, pos);
  BDevGuard dg(c->device);
  F5_CU(cudaStreamSynchronize(c->st), "set_position");
  F5_CU(cudaMemcpy(c->h_params, c->params, sizeof(StepParams) * c->B, cudaMemcpyDeviceToHost), "set_position");
  for (int b = 0; b < c->B; ++b)
    if (seq < 0 || seq == b) {
      c->h_params[b].T = T;
      c->h_params[b].pos = pos;
    }
  return cuda_status(cudaMemcpy(c->params, c->h_params, sizeof(StepParams) * c->B, cudaMemcpyHostToDevice),
                     "set_position");
}

int f5_bctx_get_position(f5_bctx *c, int seq, int *T, int *pos) {
  if (!c || seq < 0 || seq >= c->B) return set_error(F5_EINVAL, "get_position: bad sequence");
  BDevGuard dg(c->device);
  F5_CU(cudaStreamSynchronize(c->st), "get_position");
  StepParams p;
  F5_CU(cudaMemcpy(&p, c->params + seq, sizeof(p), cudaMemcpyDeviceToHost), "get_position");
  if (T) *T = p.T;
  if (pos) *pos = p.pos;
  return F5_OK;
}

int f5_bctx_step(f5_bctx *c, const int32_t *tok, int32_t *next_tok, int32_t *max_logit) {
  if (!c || !tok) return set_error(F5_EINVAL, "f5_bctx_step: null argument");
  BDevGuard dg(c->device);
  int rc = build_bgraph(c);
  if (rc) return rc;
  F5_CU(cudaStreamSynchronize(c->st), "f5_bctx_step");
  F5_CU(cudaMemcpy(c->h_params, c->params, sizeof(StepParams) * c->B, cudaMemcpyDeviceToHost), "f5_bctx_step");
  for (int b = 0; b < c->B; ++b) {
    c->h_params[b].tok = tok[b];
    c->h_params[b].err = 0;
  }
  F5_CU(cudaMemcpyAsync(c->params, c->h_params, sizeof(StepParams) * c->B, cudaMemcpyHostToDevice, c->st), "f5_bctx_step");
  F5_CU(cudaMemsetAsync(c->err, 0, 4, c->st), "f5_bctx_step");
  F5_CU(cudaGraphLaunch(c->exec, c->st), "f5_bctx_step");
  rc = bfinish(c, "f5_bctx_step");
  for (int b = 0; b < c->B; ++b) {
    if (next_tok) next_tok[b] = c->h_params[b].next_tok;
    if (max_logit) max_logit[b] = c->h_params[b].max_val;
  }
  return rc;
}

int f5_bctx_prefill(f5_bctx *c, int seq, const int32_t *tokens, int n, int32_t *next_tok, int32_t *max_logit) {
  if (!c || !tokens || n < 1) return set_error(F5_EINVAL, "f5_bctx_prefill: bad argument");
  if (seq < 0 || seq >= c->B) return set_error(F5_EINVAL, "f5_bctx_prefill: sequence %d outside [0, %d)", seq, c->B);
  BDevGuard dg(c->device);
  const int vocab = c->m->cfg.vocab;
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= vocab) return set_error(F5_EINVAL, "f5_bctx_prefill: token %d out of range", i);
  F5_CU(cudaStreamSynchronize(c->st), "f5_bctx_prefill");
  F5_CU(cudaMemcpy(c->h_params, c->params, sizeof(StepParams) * c->B, cudaMemcpyDeviceToHost), "f5_bctx_prefill");
  const int T0 = c->h_params[seq].T, pos0 = c->h_params[seq].pos;
  if (T0 + n > c->max_T) return set_error(F5_ESTATE, "f5_bctx_prefill: %d + %d tokens exceed max_T %d", T0, n, c->max_T);
  if (pos0 + n > c->m->rope_npos) return set_error(F5_ESTATE, "f5_bctx_prefill: positions past the RoPE table");
  std::vector<StepParams> pp(c->B);
  F5_CU(cudaMemsetAsync(c->err, 0, 4, c->st), "f5_bctx_prefill");
  int done = 0;
  StepParams lastp = {};
  while (done < n) {
    const int C = std::min(c->B, n - done);
    for (int t = 0; t < C; ++t) {
      pp[t] = StepParams{};
      pp[t].tok = tokens[done + t];
      pp[t].T = T0 + done + t;
      pp[t].pos = pos0 + done + t;
    }
    F5_CU(cudaMemcpyAsync(c->pparams, pp.data(), sizeof(StepParams) * C, cudaMemcpyHostToDevice, c->st),
          "f5_bctx_prefill");
    const bool last = done + C == n;
    cudaError_t e = enqueue_prefill_chunk(c, seq, C, last);
    c->ncol = 0;
    if (e != cudaSuccess) return cuda_status(e, "f5_bctx_prefill");
    // pp is reused by the next chunk's copy: wait for this chunk first
    F5_CU(cudaStreamSynchronize(c->st), "f5_bctx_prefill");
    if (last) F5_CU(cudaMemcpy(&lastp, c->pparams + (C - 1), sizeof(lastp), cudaMemcpyDeviceToHost), "f5_bctx_prefill");
    done += C;
  }
  uint32_t herr = 0;
  F5_CU(cudaMemcpy(&herr, c->err, 4, cudaMemcpyDeviceToHost), "f5_bctx_prefill");
  c->h_params[seq].T = T0 + n;
  c->h_params[seq].pos = pos0 + n;
  c->h_params[seq].next_tok = lastp.next_tok;
  c->h_params[seq].max_val = lastp.max_val;
  c->h_params[seq].tok = lastp.next_tok;
  F5_CU(cudaMemcpy(c->params, c->h_params, sizeof(StepParams) * c->B, cudaMemcpyHostToDevice), "f5_bctx_prefill");
  if (next_tok) *next_tok = lastp.next_tok;
  if (max_logit) *max_logit = lastp.max_val;
  if ((herr | lastp.err) & DERR_TIMEOUT) return set_error(F5_ETIMEOUT, "f5_bctx_prefill: a bounded device wait expired");
  if ((herr | lastp.err) & DERR_Y32_OVERFLOW) return set_error(F5_EOVERFLOW, "f5_bctx_prefill: |y32| >= 2^31");
  if ((herr | lastp.err) & DERR_KV_FULL) return set_error(F5_ESTATE, "f5_bctx_prefill: KV cache full (max_T)");
  if ((herr | lastp.err) & DERR_RANGE) return set_error(F5_EINVAL, "f5_bctx_prefill: input out of range");
  return F5_OK;
}

int f5_bctx_launch(f5_bctx *c, int n_steps) {
  if (!c || n_steps < 0) return set_error(F5_EINVAL, "f5_bctx_launch: bad argument");
  BDevGuard dg(c->device);
  int rc = build_bgraph(c);
  if (rc) return rc;
  for (int i = 0; i < n_steps; ++i) F5_CU(cudaGraphLaunch(c->exec, c->st), "f5_bctx_launch");
  return F5_OK;
}

int f5_bctx_sync(f5_bctx *c, int32_t *last_tok, int32_t *max_logit) {
  if (!c) return set_error(F5_EINVAL, "null batched context");
  BDevGuard dg(c->device);
  int rc = bfinish(c, "f5_bctx_sync");
  for (int b = 0; b < c->B; ++b) {
    if (last_tok) last_tok[b] = c->h_params[b].next_tok;
    if (max_logit) max_logit[b] = c->h_params[b].max_val;
  }
  return rc;
}

int f5_bctx_time_step(f5_bctx *c, int reps, double *out, int nout) {
  if (!c || !out || nout < 2 * BK_N + 2 || reps < 1) return set_error(F5_EINVAL, "f5_bctx_time_step: bad argument");
  BDevGuard dg(c->device);
  double ms[BK_N] = {}, bytes[BK_N] = {};
  double launches = 0;
  for (int r = 0; r < reps; ++r) {
    c->timing = true;
    c->timed.clear();
    cudaError_t e = enqueue_bstep(c);
    c->timing = false;
    if (e != cudaSuccess) return cuda_status(e, "f5_bctx_time_step");
    F5_CU(cudaStreamSynchronize(c->st), "f5_bctx_time_step");
    for (f5_bctx::Timed &t : c->timed) {
      float x = 0;
      cudaEventElapsedTime(&x, t.a, t.b);
      ms[t.kind] += x / reps;
      bytes[t.kind] += t.bytes / reps;
      cudaEventDestroy(t.a);
      cudaEventDestroy(t.b);
    }
    launches = (double)c->timed.size() + 2;
    c->timed.clear();
  }
  for (int k = 0; k < BK_N; ++k) {
    out[k] = ms[k];
    out[BK_N + k] = bytes[k];
  }
  out[2 * BK_N] = launches;
  out[2 * BK_N + 1] = 0;
  for (int k = 0; k < BK_N; ++k) out[2 * BK_N + 1] += ms[k];
  return bfinish(c, "f5_bctx_time_step");
}

int f5_bctx_set_logits(f5_bctx *c, int on) {
  if (!c) return set_error(F5_EINVAL, "null batched context");
  BDevGuard dg(c->device);
  if (on && !c->logits) {
    int rc = balloc(c, reinterpret_cast<void **>(&c->logits), (size_t)c->B * c->m->cfg.vocab * 4);
    if (rc) return rc;
  }
  if ((on != 0) != c->want_logits) {
    c->want_logits = on != 0;
    c->dirty = true;   // the step graph is recorded again with the LM head's y32 output
  }
  return F5_OK;
}

int f5_bctx_topk(f5_bctx *c, f5_topk32 *out) {
  if (!c || !out) return set_error(F5_EINVAL, "null argument");
  if (!c->logits || !c->want_logits)
    return set_error(F5_ESTATE, "f5_bctx_topk: logits not stored (f5_bctx_set_logits(bctx, 1) before the step)");
  BDevGuard dg(c->device);
  const int vocab = c->m->cfg.vocab;
  int rc;
  if (!c->tk_ws) {
    if ((rc = balloc(c, &c->tk_ws, (size_t)c->B * topk32_ws_bytes(vocab)))) return rc;
    if ((rc = balloc(c, reinterpret_cast<void **>(&c->tk_out), (size_t)c->B * sizeof(f5_topk32)))) return rc;
  }
  // the LM head's prologue left each sequence's {e_x, in_f} in xmeta
  F5_CU(launch_topk32_b(c->logits, vocab, c->B, vocab, c->tk_ws, c->tk_out, c->xmeta, 2, c->st), "f5_bctx_topk");
  F5_CU(cudaMemcpyAsync(out, c->tk_out, (size_t)c->B * sizeof(f5_topk32), cudaMemcpyDeviceToHost, c->st),
        "f5_bctx_topk");
  F5_CU(cudaStreamSynchronize(c->st), "f5_bctx_topk");
  return F5_OK;
}

int f5_bctx_stream(f5_bctx *c, void **stream) {
  if (!c || !stream) return set_error(F5_EINVAL, "null argument");
  *stream = c->st;
  return F5_OK;
}

int f5_bctx_read(f5_bctx *c, int seq, int what, int layer, void *dst, size_t bytes) {
  if (!c || !dst) return set_error(F5_EINVAL, "null argument");
  BDevGuard dg(c->device);
  uint8_t *p;
  size_t n;
  int rc = bbuf(c, what, layer, seq, &p, &n);
  if (rc) return rc;
  if (bytes != n) return set_error(F5_EINVAL, "f5_bctx_read: %zu bytes, buffer holds %zu", bytes, n);
  F5_CU(cudaStreamSynchronize(c->st), "f5_bctx_read");
  return cuda_status(cudaMemcpy(dst, p, n, cudaMemcpyDeviceToHost), "f5_bctx_read");
}

int f5_bctx_write(f5_bctx *c, int seq, int what, int layer, const void *src, size_t bytes) {
  if (!c || !src) return set_error(F5_EINVAL, "null argument");
  BDevGuard dg(c->device);
  uint8_t *p;
  size_t n;
  int rc = bbuf(c, what, layer, seq, &p, &n);
  if (rc) return rc;
  if (bytes != n) return set_error(F5_EINVAL, "f5_bctx_write: %zu bytes, buffer holds %zu", bytes, n);
  F5_CU(cudaStreamSynchronize(c->st), "f5_bctx_write");
  return cuda_status(cudaMemcpy(p, src, n, cudaMemcpyHostToDevice), "f5_bctx_write");
}

}  // extern "C"
