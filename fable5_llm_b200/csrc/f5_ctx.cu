// Model context: one GPU's resident 9B integer model, its decode state and
// the decode step in two engines.
//
// Replaces the reference's model-level step (ref/fidelity_check.py:404-448
// FxRunner.step; ref/gen_model_script.py:602-650 token loop) and, for one
// layer, ref/layer_fixed.py:1669-1677 layer_decode_fx.  The 39k-record SEQ
// program the FPGA sequencer runs per token is replaced by
//  * F5_ENGINE_PERSISTENT: one cooperative launch of the persistent decode
//    kernel (f5_mega.cu) walking a device-resident list of op descriptors;
//  * F5_ENGINE_GRAPH: a fixed chain of 163 kernel launches (step begin, 5
//    per layer, LM head, step end) recorded once into a CUDA graph with
//    programmatic dependent launch edges.
// Both are built by the same enqueue_step walk (the persistent program is
// the walk in "emit" mode), so they run the same descriptors.
#include <algorithm>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/f5b200.h"
#include "f5_attn.cuh"
#include "f5_capi_util.h"
#include "f5_dn.cuh"
#include "f5_int.cuh"
#include "f5_kernels.cuh"
#include "f5_mega.cuh"
#include "f5_batch.cuh"
#include "f5_topk.cuh"

namespace f5 {
cudaError_t launch_synth_w4(uint8_t *, long long, int, int, long long, uint64_t, uint64_t, int, cudaStream_t);
cudaError_t launch_synth_emb(int16_t *, long long, int, long long, uint64_t, cudaStream_t);

// step begin: x16 = emb[tok] (ref/fidelity_check.py:428), reset argmax key
__global__ void k_step_begin(StepParams *p, const int16_t *emb, int vocab, int H, int16_t *x16,
                             unsigned long long *key) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int tok = p->tok;
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(&p->err, DERR_RANGE);
    tok = 0;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x)
    x16[i] = emb[(size_t)tok * H + i];
  if (blockIdx.x == 0 && threadIdx.x == 0) *key = 0ull;
}

// step end: decode the argmax key; feed the token back for a greedy loop
__global__ void k_step_end(StepParams *p, const unsigned long long *key, const uint32_t *err, int advance) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const unsigned long long k = *key;
  const int row = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
  const int val = (int)((uint32_t)(k >> 32) ^ 0x80000000u);
  p->next_tok = row;
  p->max_val = val;
  p->err |= *err;
  if (advance) {
    p->tok = row;
    p->pos += 1;
    p->T += 1;
    p->steps += 1;
  }
}

__global__ void k_collect_err(StepParams *p, const uint32_t *err) { p->err |= *err; }

// prefill: the input token of the next step comes from the prompt, not the argmax
__global__ void k_set_token(StepParams *p, const int32_t *toks, int i) { p->tok = toks[i]; }

static cudaError_t launch_pdl(const void *fn, void **args, dim3 grid, dim3 block, cudaStream_t st, bool pdl) {
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

}  // namespace f5

#include "f5_ctx_priv.h"

namespace f5 {

static int alloc(f5_ctx *c, void **p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaMalloc");
  c->allocs.push_back(*p);
  e = cudaMemsetAsync(*p, 0, bytes, c->st);
  return cuda_status(e, "cudaMemset");
}
#define F5_ALLOC(c, p, bytes)                                          \
  do {                                                                 \
    int _rc = alloc((c), reinterpret_cast<void **>(&(p)), (bytes));    \
    if (_rc) return _rc;                                               \
  } while (0)
#define F5_CU(x, what)                        \
  do {                                        \
    int _rc = cuda_status((x), (what));       \
    if (_rc) return _rc;                      \
  } while (0)

struct DevGuard {
  int prev = 0;
  explicit DevGuard(int d) { cudaGetDevice(&prev); cudaSetDevice(d); }
  ~DevGuard() { cudaSetDevice(prev); }
};

enum { TK_GEMV = 0, TK_DN = 1, TK_ATTN = 2, TK_OTHER = 3 };
static void tl_begin(f5_ctx *c) {
  if (!c->timing) return;
  f5_ctx::Timed t = {};
  cudaEventCreate(&t.a);
  cudaEventCreate(&t.b);
  cudaEventRecord(t.a, c->st);
  c->timed.push_back(t);
}
static void tl_end(f5_ctx *c, int kind, double bytes) {
  if (!c->timing) return;
  f5_ctx::Timed &t = c->timed.back();
  t.kind = kind;
  t.bytes = bytes;
  cudaEventRecord(t.b, c->st);
}

static void split_rows(int n, int ws, int rank, int &r0, int &cnt) {
  const int base = n / ws, rem = n % ws;
  r0 = rank * base + (rank < rem ? rank : rem);
  cnt = base + (rank < rem ? 1 : 0);
}

static DevMat *find_mat(f5_ctx *c, int layer, int slot) {
  if (layer == -1) return slot == 0 ? &c->head : nullptr;
  if (layer < 0 || layer >= (int)c->L.size() || slot < 0 || slot >= NSLOT) return nullptr;
  return &c->L[layer].m[slot];
}

static bool slot_valid(const Layer &l, int slot) {
  if (slot >= 8 && slot <= 10) return true;
  return l.attn ? slot <= 3 : slot <= 4;
}

static void expected_shape(const f5_ctx *c, int layer, int slot, int &N, int &K) {
  N = K = 0;
  if (layer == -1) { N = c->cfg.vocab; K = H; return; }
  const bool attn = c->L[layer].attn;
  switch (slot) {
    case 8: case 9: N = FFN; K = H; return;
    case 10: N = H; K = FFN; return;
    default: break;
  }
  if (attn) {
    const int n[4] = {NQ * HD * 2, NKV * HD, NKV * HD, H}, k[4] = {H, H, H, NQ * HD};
    N = n[slot]; K = k[slot];
  } else {
    const int n[5] = {CONV_DIM, LVD, LNH, LNH, H}, k[5] = {H, H, H, H, LVD};
    N = n[slot]; K = k[slot];
  }
}

static int prep_matrix(f5_ctx *c, int layer, int slot, int N, int K, int g, int e, int sh, DevMat *&m) {
  m = find_mat(c, layer, slot);
  if (!m || (layer >= 0 && !slot_valid(c->L[layer], slot)))
    return set_error(F5_EINVAL, "no matrix slot %d in layer %d", slot, layer);
  int eN, eK;
  expected_shape(c, layer, slot, eN, eK);
  if (N != eN || K != eK) return set_error(F5_EINVAL, "layer %d slot %d: shape %dx%d, expected %dx%d", layer, slot, N, K, eN, eK);
  int st = check_matrix_shape(N, K, g);
  if (st) return st;
  if (g != 128) return set_error(F5_EINVAL, "the decode step uses g=128 images");
  if (sh != (int)(64 - __builtin_clzll((unsigned long long)(K / g) * 65535ull * (unsigned long long)(g * 8 * 127))) - 31)
    return set_error(F5_EINVAL, "sh=%d is not the final shift of K=%d (ref/w4a8_ref.py:177-179)", sh, K);
  m->N = N; m->K = K; m->g = g; m->e = e; m->sh = sh; m->stride = row_stride(K, g);
  split_rows(N, c->cfg.world_size, c->cfg.rank, m->row0, m->rows);
  if (!m->w) F5_ALLOC(c, m->w, (size_t)m->rows * m->stride + 64);
  c->graph_dirty = c->mega_dirty = true;
  return F5_OK;
}

static int check_ctx(f5_ctx *c) {
  if (!c) return set_error(F5_EINVAL, "null context");
  return F5_OK;
}

static GemvSeg mkseg(const DevMat &m, void *out, int mode, int out_f, const DevMat *m2 = nullptr, int out_f2 = 0) {
  GemvSeg s = {};
  s.w = m.w;
  s.w2 = m2 ? m2->w : nullptr;
  s.out = out;
  s.rows = m.rows;
  s.e = m.e;
  s.e2 = m2 ? m2->e : 0;
  s.out_f = out_f;
  s.out_f2 = out_f2;
  s.mode = mode;
  s.out_row0 = m.row0;
  return s;
}

// Ops whose inputs are all dataflow-tagged run without a grid barrier; the
// op after BEGIN (which also clears the step's slots and sums) and the
// attention out-projection (its input sums are atomics) take one.
static void emit_op(f5_ctx *c, MegaOp &op, bool need_bar) {
  op.bar = need_bar ? c->emit_nbar++ : -1;
  c->emit->push_back(op);
}

// the tagged twin of a plain activation pointer (nullptr if none)
static f5_ctx::Twin *twin_of(f5_ctx *c, const void *p, uint32_t **tp) {
  for (f5_ctx::Twin &t : c->twins) {
    const char *b = static_cast<const char *>(t.plain), *q = static_cast<const char *>(p);
    if (q >= b && q < b + t.plain_bytes) {
      if (tp) *tp = t.tagged + (q - b) / t.elem;
      return &t;
    }
  }
  return nullptr;
}
// writer side: route a segment's output to the twin, tagged by op index idx
static void tag_output(f5_ctx *c, void *&out, int idx) {
  uint32_t *tp;
  f5_ctx::Twin *t = twin_of(c, out, &tp);
  if (!t) return;
  out = tp;
  t->last_op1 = idx + 1;
}
// reader side: route an input to the twin; returns its writer's tag (op1)
template <class P>
static int tag_input(f5_ctx *c, P *&in) {
  uint32_t *tp;
  f5_ctx::Twin *t = twin_of(c, in, &tp);
  if (!t) return 0;
  in = reinterpret_cast<P *>(tp);
  return t->last_op1;
}

static cudaError_t gemv(f5_ctx *c, const GemvSeg *segs, int nseg, int K, const GemvPrologue &pro,
                        unsigned long long *key, bool pdl) {
  GemvArgs a = {};
  int units = 0;
  for (int i = 0; i < nseg; ++i) {
    a.seg[i] = segs[i];
    a.seg[i].unit_begin = units;
    units += segs[i].rows;
  }
  a.nseg = nseg;
  a.total_units = units;
  a.K = K;
  a.g = 128;
  a.stride = row_stride(K, 128);
  a.sh = (int)(64 - __builtin_clzll((unsigned long long)(K / 128) * 65535ull * 130048ull)) - 31;
  a.pro = pro;
  a.argmax_key = key;
  a.err = c->err;
  double bytes = 0;
  for (int i = 0; i < nseg; ++i) bytes += (double)segs[i].rows * a.stride * (segs[i].mode == GM_SILU_MUL ? 2 : 1);
  if (c->emit) {
    // persistent program: same descriptor, ring-stage chunking, one CTA per SM
    a.rows_per_stage = mega_rows_per_stage(a.stride);
    a.stages = 0;
    bool paired = false, argmax = false;
    for (int i = 0; i < nseg; ++i) {
      paired |= segs[i].mode == GM_SILU_MUL;
      argmax |= segs[i].mode == GM_ARGMAX;
    }
    const int per_cta = (units + c->mega_grid - 1) / c->mega_grid;
    // K = 12288 rows are reduced as 3 K-parts by 15 warps: <= 5 rows per stage
    if (K == 12288 && a.rows_per_stage > 5) a.rows_per_stage = 5;
    const int res_per_unit = paired ? 2 : (K == 12288 ? 3 : 1);
    if ((K != 4096 && K != 12288) || (argmax && (nseg != 1 || K != 4096)) || pro.mode == PRO_X8 ||
        (K == 12288 && (paired || argmax)) || (!argmax && per_cta * res_per_unit > MEGA_RES) ||
        a.rows_per_stage < 2)
      c->emit_err = 1;
    // dataflow tags: the prologue's input from its twin (tagged by its last
    // writer), then this op's outputs to their twins
    const int idx = (int)c->emit->size();
    if (a.pro.mode == PRO_RMSNORM || a.pro.mode == PRO_DYNQ8) a.pro.tag_op1 = tag_input(c, a.pro.src);
    else if (a.pro.mode == PRO_ATTN_ACC) a.pro.tag_op1 = tag_input(c, a.pro.src2);
    for (int i = 0; i < nseg; ++i) {
      GemvSeg &sg = a.seg[i];
      switch (sg.mode) {
        case GM_TO16: case GM_RESID: case GM_SILU_MUL:
          if (twin_of(c, sg.out, nullptr)) { tag_output(c, sg.out, idx); sg.tag_op1 = idx + 1; }
          break;
        case GM_CONV: case GM_GATE_B: case GM_GATE_A:
          if (twin_of(c, sg.aux_out, nullptr)) { tag_output(c, sg.aux_out, idx); sg.tag_op1 = idx + 1; sg.out = nullptr; }
          break;
        default: break;
      }
    }
    MegaOp op = {};
    op.kind = MK_GEMV;
    op.g = a;
    emit_op(c, op, idx == 1 || a.pro.mode == PRO_ATTN_ACC);
    return cudaSuccess;
  }
  tl_begin(c);
  cudaError_t e = launch_gemv(a, c->st, pdl, sm_count());
  tl_end(c, TK_GEMV, bytes);
  return e;
}

// per attention layer of the persistent program: marked exchange slots
// [2 phases][NKV][cpg][4 heads][2 words] (u64) and the PV sums [NQ*HD] (i32)
static size_t att_acc_bytes(int cpg) { return (size_t)2 * NKV * cpg * 4 * 2 * 8 + (size_t)NQ * HD * 4; }
static size_t n_attn_layers(const f5_ctx *c) {
  size_t n = 0;
  for (const Layer &l : c->L) n += l.attn ? 1 : 0;
  return n;
}
// per DeltaNet layer of the persistent program: marked o values [LNH][128][2] (u64)
constexpr size_t DN_XSLOT_BYTES = (size_t)LNH * 128 * 2 * 8;
// the per-step zeroed region: attention layers first, then DeltaNet layers
static size_t step_acc_bytes(const f5_ctx *c, int cpg) {
  return n_attn_layers(c) * att_acc_bytes(cpg) + (c->L.size() - n_attn_layers(c)) * DN_XSLOT_BYTES;
}

// the five launches of one layer (ref/layer_fixed.py:1669-1677)
static cudaError_t enqueue_layer(f5_ctx *c, int li, bool pdl) {
  Layer &l = c->L[li];
  cudaError_t e;
  GemvPrologue pro = {};
  pro.mode = PRO_RMSNORM;
  pro.src = c->x16;
  pro.w = l.ln1;
  pro.in_f = RS_F;
  pro.one_plus = 1;
  if (!l.attn) {
    // in-projection: qkv16 (Q.RS_F), z16 (Q.QKV_F), b, a (Q12), ref/layer_fixed.py:1503-1509,
    // with conv4+SiLU per channel and the two gates per head in the epilogues
    GemvSeg s[4] = {mkseg(l.m[0], c->qkv16, GM_CONV, RS_F), mkseg(l.m[1], c->z16, GM_TO16, QKV_F),
                    mkseg(l.m[2], c->b16, GM_GATE_B, 12), mkseg(l.m[3], c->a16, GM_GATE_A, 12)};
    s[0].aux_out = c->qkvc16;
    s[0].aux0 = l.conv;
    s[0].aux1 = l.conv_w;
    s[0].T = &c->params->T;
    s[2].aux_out = c->gates;
    s[3].aux_out = c->gates + LNH;
    s[3].aux0 = l.dt_bias;
    s[3].aux1 = l.A;
    if ((e = gemv(c, s, 4, H, pro, nullptr, pdl))) return e;
    DnArgs d = {};
    d.qkvc = c->qkvc16; d.beta = c->gates; d.decay = c->gates + LNH; d.z16 = c->z16; d.norm_w = l.norm_w;
    d.S = l.S; d.on16 = c->on16; d.kh_out = l.kh; d.stats = c->stats; d.err = c->err;
    d.lkd = LKD; d.vrep = LNH / LNKH; d.norm_mode = c->cfg.norm_mode;
    if (c->emit) {
      const int n_dn = (int)std::count_if(c->emit->begin(), c->emit->end(),
                                          [](const MegaOp &o) { return o.kind == MK_DN; });
      d.xslots = reinterpret_cast<unsigned long long *>(
          reinterpret_cast<uint8_t *>(c->d_attacc) + n_attn_layers(c) * att_acc_bytes(c->mega_grid / NKV) +
          (size_t)n_dn * DN_XSLOT_BYTES);
      const int idx = (int)c->emit->size();
      d.in_tag_op1 = tag_input(c, d.qkvc);
      tag_input(c, d.z16);
      tag_input(c, d.beta);
      tag_input(c, d.decay);
      void *on = d.on16;
      tag_output(c, on, idx);
      if (on != (void *)d.on16) {
        d.on16 = static_cast<int16_t *>(on);
        d.out_tag_op1 = idx + 1;
      }
      MegaOp op = {};
      op.kind = MK_DN;
      op.d = d;
      emit_op(c, op, false);
    } else {
      tl_begin(c);
      e = launch_dn_step(d, LNH, c->st, pdl);
      tl_end(c, TK_DN, 0);
      if (e) return e;
    }
    GemvPrologue p2 = {};
    p2.mode = PRO_DYNQ8;
    p2.src = c->on16;
    p2.in_f = DN_NORM_F;
    GemvSeg so = mkseg(l.m[4], c->x16, GM_RESID, RS_F);
    if ((e = gemv(c, &so, 1, LVD, p2, nullptr, pdl))) return e;
  } else {
    GemvSeg s[3] = {mkseg(l.m[0], c->qg16, GM_TO16, QKV_F), mkseg(l.m[1], c->k16, GM_TO16, QKV_F),
                    mkseg(l.m[2], c->v16, GM_TO16, QKV_F)};
    if ((e = gemv(c, s, 3, H, pro, nullptr, pdl))) return e;
    AttnArgs at = {};
    at.qg16 = c->qg16; at.k16 = c->k16; at.v16 = c->v16; at.q_norm = l.q_norm; at.k_norm = l.k_norm;
    at.rope = c->rope; at.k8 = l.k8; at.ke = l.ke; at.v8 = l.v8; at.ve = l.ve; at.prod = c->prod64;
    at.T = &c->params->T; at.pos = &c->params->pos; at.err = c->err;
    at.max_T = c->cfg.max_T; at.max_pos = c->rope_npos; at.nq = NQ; at.nkv = NKV; at.rot = ROT;
    GemvPrologue p2 = {};
    p2.mode = PRO_ATTN_GATE;
    p2.src = c->prod64;
    p2.dbg = l.ka;
    if (c->emit) {
      // split-T over G/NKV CTAs per KV head; sums land in this layer's accumulators
      const int n_attn = (int)std::count_if(c->emit->begin(), c->emit->end(),
                                            [](const MegaOp &o) { return o.kind == MK_ATTN; });
      const int cpg = c->mega_grid / NKV;
      uint8_t *acc = reinterpret_cast<uint8_t *>(c->d_attacc) + (size_t)n_attn * att_acc_bytes(cpg);
      MegaOp op = {};
      op.kind = MK_ATTN;
      op.at.a = at;
      op.at.a.chunk_max = (((c->cfg.max_T + cpg - 1) / cpg) + 15) & ~15;
      op.at.slots = reinterpret_cast<unsigned long long *>(acc);
      op.at.gacc = reinterpret_cast<int32_t *>(acc + (size_t)2 * NKV * cpg * 4 * 2 * 8);
      op.at.in_tag_op1 = tag_input(c, op.at.a.qg16);
      tag_input(c, op.at.a.k16);
      tag_input(c, op.at.a.v16);
      emit_op(c, op, false);
      p2.mode = PRO_ATTN_ACC;
      p2.src = op.at.gacc;
      p2.src2 = c->qg16;
    } else {
      tl_begin(c);
      e = launch_attn(at, c->st, pdl);
      tl_end(c, TK_ATTN, 0);
      if (e) return e;
    }
    GemvSeg so = mkseg(l.m[3], c->x16, GM_RESID, RS_F);
    if ((e = gemv(c, &so, 1, NQ * HD, p2, nullptr, pdl))) return e;
  }
  // MLP (ref/layer_fixed.py:1597-1604) with both residual adds fused
  GemvPrologue p3 = {};
  p3.mode = PRO_RMSNORM;
  p3.src = c->x16;
  p3.w = l.ln2;
  p3.in_f = RS_F;
  p3.one_plus = 1;
  GemvSeg sgu = mkseg(l.m[8], c->prod16, GM_SILU_MUL, 12, &l.m[9], RS_F);
  if ((e = gemv(c, &sgu, 1, H, p3, nullptr, pdl))) return e;
  GemvPrologue p4 = {};
  p4.mode = PRO_DYNQ8;
  p4.src = c->prod16;
  p4.in_f = RS_F;
  GemvSeg sd = mkseg(l.m[10], c->x16, GM_RESID, RS_F);
  sd.rstat = c->stats + 1;   // the layer output: FxRunner's resid_max / resid_clip
  return gemv(c, &sd, 1, FFN, p4, nullptr, pdl);
}

static cudaError_t enqueue_step(f5_ctx *c, bool pdl) {
  cudaError_t e;
  if (c->emit) {
    MegaOp op = {};
    op.kind = MK_BEGIN;
    op.b.emb = c->emb;
    op.b.x16 = c->x16;
    op.b.vocab = c->cfg.vocab;
    op.b.H = H;
    op.b.key = c->key;
    op.b.zero = c->d_attacc;
    op.b.zero_n = (int)(step_acc_bytes(c, c->mega_grid / NKV) / 16);
    void *xt = c->x16;
    tag_output(c, xt, 0);   // BEGIN writes the tagged residual as op 0
    op.b.x16t = xt != (void *)c->x16 ? static_cast<uint32_t *>(xt) : nullptr;
    emit_op(c, op, false);
  } else {
    StepParams *p = c->params;
    const int16_t *emb = c->emb;
    int vocab = c->cfg.vocab, h = H;
    int16_t *x = c->x16;
    unsigned long long *k = c->key;
    void *args[] = {&p, &emb, &vocab, &h, &x, &k};
    tl_begin(c);
    e = launch_pdl((const void *)k_step_begin, args, dim3(4), dim3(256), c->st, pdl);
    tl_end(c, TK_OTHER, 0);
    if (e) return e;
  }
  for (int li = 0; li < (int)c->L.size(); ++li)
    if ((e = enqueue_layer(c, li, pdl))) return e;
  GemvPrologue pf = {};
  pf.mode = PRO_RMSNORM;
  pf.src = c->x16;
  pf.w = c->ln_f;
  pf.in_f = RS_F;
  pf.one_plus = 0;   // ln_f pre-folded (1+w) at Q3.12 (ref/gen_model_script.py:502-504)
  GemvSeg sh = mkseg(c->head, c->want_logits ? c->logits : nullptr, GM_ARGMAX, 0);
  if ((e = gemv(c, &sh, 1, H, pf, c->key, pdl))) return e;
  if (!c->emit) {
    StepParams *p = c->params;
    const unsigned long long *k = c->key;
    const uint32_t *er = c->err;
    int adv = 1;
    void *args[] = {&p, &k, &er, &adv};
    tl_begin(c);
    e = launch_pdl((const void *)k_step_end, args, dim3(1), dim3(1), c->st, pdl);
    tl_end(c, TK_OTHER, 0);
    if (e) return e;
  }
  return cudaSuccess;
}

static int layer_ready(f5_ctx *c, int li) {
  for (int s = 0; s < NSLOT; ++s)
    if (slot_valid(c->L[li], s) && !c->L[li].m[s].w)
      return set_error(F5_ESTATE, "layer %d slot %d not uploaded", li, s);
  if (!c->rope) return set_error(F5_ESTATE, "RoPE table not uploaded");
  return F5_OK;
}

static int ready(f5_ctx *c) {
  for (size_t i = 0; i < c->L.size(); ++i)
    for (int s = 0; s < NSLOT; ++s)
      if (slot_valid(c->L[i], s) && !c->L[i].m[s].w)
        return set_error(F5_ESTATE, "layer %zu slot %d not uploaded", i, s);
  if (!c->head.w) return set_error(F5_ESTATE, "LM head not uploaded");
  if (!c->emb) return set_error(F5_ESTATE, "embedding not uploaded");
  if (!c->rope) return set_error(F5_ESTATE, "RoPE table not uploaded");
  return F5_OK;
}

static int build_graph(f5_ctx *c) {
  if (!c->graph_dirty && c->step_exec) return F5_OK;
  int rc = ready(c);
  if (rc) return rc;
  if (c->cfg.world_size > 1)
    return set_error(F5_ESTATE, "row-sharded contexts need an output all-gather (f5_ctx_attach_comm) before decoding");
  if (c->step_exec) {
    cudaGraphExecDestroy(c->step_exec);
    c->step_exec = nullptr;
  }
  F5_CU(cudaStreamSynchronize(c->st), "sync before capture");
  cudaGraph_t g = nullptr;
  F5_CU(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal), "begin capture");
  cudaError_t e = enqueue_step(c, true);
  cudaError_t e2 = cudaStreamEndCapture(c->st, &g);
  if (e != cudaSuccess) { if (g) cudaGraphDestroy(g); return cuda_status(e, "capture decode step"); }
  F5_CU(e2, "end capture");
  e = cudaGraphInstantiate(&c->step_exec, g, 0);
  cudaGraphDestroy(g);
  F5_CU(e, "instantiate decode graph");
  c->graph_dirty = false;
  return F5_OK;
}

// The dataflow-tagged twins of the activations the persistent program passes
// between ops, plus the cross-rank argmax key slots, in ONE allocation (one
// CUDA IPC handle per rank; the layout is identical on every rank).
static int ensure_twins(f5_ctx *c) {
  if (c->twin_mem) return F5_OK;
  struct { void *p; size_t bytes, elem; } tw[] = {
      {c->x16, H * 2, 2}, {c->qkvc16, CONV_DIM * 2, 2}, {c->z16, LVD * 2, 2}, {c->gates, 2 * LNH * 4, 4},
      {c->on16, LVD * 2, 2}, {c->prod16, FFN * 2, 2}, {c->qg16, NQ * HD * 2 * 2, 2}, {c->k16, NKV * HD * 2, 2},
      {c->v16, NKV * HD * 2, 2}};
  size_t words = 0;
  for (auto &t : tw) words += t.bytes / t.elem;
  words = (words + 3) & ~(size_t)3;   // 16-byte aligned key slots
  const size_t key_bytes = (size_t)F5_MAX_RANKS * 2 * 8;
  F5_ALLOC(c, c->twin_mem, words * 4 + key_bytes);
  c->twin_bytes = words * 4 + key_bytes;
  c->xkey = reinterpret_cast<unsigned long long *>(c->twin_mem + words);
  words = 0;
  for (auto &t : tw) {
    c->twins.push_back({t.p, t.bytes, t.elem, c->twin_mem + words, 0});
    words += t.bytes / t.elem;
  }
  return F5_OK;
}

static void free_mega(f5_ctx *c) {
  if (c->d_ops) cudaFree(c->d_ops);
  if (c->d_bars) cudaFree(c->d_bars);
  c->d_ops = nullptr;
  c->d_bars = nullptr;
}

// Emit the step as the persistent kernel's op list.  `unsupported` tells a
// configuration the persistent engine cannot run (auto mode then uses the
// graph engine) from a context that is not ready.
static int build_mega(f5_ctx *c, bool &unsupported) {
  unsupported = false;
  if (!c->mega_dirty && c->d_ops) return F5_OK;
  int rc = ready(c);
  if (rc) return rc;
  unsupported = true;
  if (c->cfg.world_size > 1 && !c->peers_attached)
    return set_error(F5_ESTATE, "row-sharded context: exchange IPC handles (f5_ctx_ipc_handle / f5_ctx_attach_peers) first");
  if (c->cfg.world_size > F5_MAX_RANKS) return set_error(F5_EINVAL, "at most %d ranks", F5_MAX_RANKS);
  const int sms = sm_count();
  if (sms < 4 * LNH) return set_error(F5_ESTATE, "the persistent engine needs >= %d SMs", 4 * LNH);
  const int cpg = sms / NKV;
  const int chunk_max = (((c->cfg.max_T + cpg - 1) / cpg) + 15) & ~15;
  int grid = 0, ns = 0;
  size_t smem = 0;
  cudaError_t e = mega_config(chunk_max, &grid, &smem, &ns);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(F5_ESTATE, "persistent engine not resident on this device: %s", cudaGetErrorString(e));
  }
  c->mega_grid = grid;
  c->mega_smem = smem;
  const size_t n_attn = n_attn_layers(c);
  if (!c->d_attacc) {
    unsupported = false;
    F5_ALLOC(c, c->d_attacc, step_acc_bytes(c, cpg) + 16);
    unsupported = true;
  }
  unsupported = false;
  if ((rc = ensure_twins(c))) return rc;
  unsupported = true;
  for (f5_ctx::Twin &t : c->twins) t.last_op1 = 0;
  std::vector<MegaOp> ops;
  c->emit = &ops;
  c->emit_err = 0;
  c->emit_nbar = 0;
  e = enqueue_step(c, false);
  c->emit = nullptr;
  if (e != cudaSuccess) return cuda_status(e, "emit persistent program");
  if (c->emit_err) return set_error(F5_ESTATE, "a GEMV of this model does not fit the persistent engine");
  if (ops.size() > 256) return set_error(F5_ESTATE, "persistent program of %zu ops (dataflow tags index < 256)", ops.size());
  const int nbars = c->emit_nbar + 2;   // grid barriers, abort flag, final arrivals
  for (MegaOp &op : ops)
    if (op.kind == MK_GEMV) op.g.abort_flag = nullptr;   // patched below once the barrier array exists
  unsupported = false;
  free_mega(c);
  F5_CU(cudaMalloc(&c->d_ops, ops.size() * sizeof(MegaOp)), "persistent program");
  F5_CU(cudaMalloc(&c->d_bars, (size_t)nbars * 4), "persistent barriers");
  for (MegaOp &op : ops) {
    if (op.kind == MK_GEMV) {
      op.g.abort_flag = c->d_bars + nbars - 2;
      op.g.nrank = c->cfg.world_size;
      for (int r = 0; r < F5_MAX_RANKS; ++r) op.g.peer_delta[r] = c->peer_delta[r];
    } else if (op.kind == MK_BEGIN) {
      // this rank's rows of the 4096-row residual GEMVs (every layer's out /
      // o_proj / down matrix splits N = 4096 the same way)
      const DevMat &dm = c->L[0].m[c->L[0].attn ? 3 : 4];
      op.b.res_row0 = dm.row0;
      op.b.res_rows = dm.rows;
    }
  }
  F5_CU(cudaMemcpyAsync(c->d_ops, ops.data(), ops.size() * sizeof(MegaOp), cudaMemcpyHostToDevice, c->st),
        "persistent program");
  F5_CU(cudaMemsetAsync(c->d_bars, 0, (size_t)nbars * 4, c->st), "persistent barriers");
  F5_CU(cudaStreamSynchronize(c->st), "persistent program");
  MegaArgs &m = c->margs;
  m = {};
  m.ops = c->d_ops;
  m.nops = (int)ops.size();
  m.params = c->params;
  m.bars = c->d_bars;
  m.nbars = nbars;
  m.err = c->err;
  m.advance = 1;
  m.dn_heads = LNH;
  m.ns = ns;
  m.nrank = c->cfg.world_size;
  m.rank = c->cfg.rank;
  for (int r = 0; r < F5_MAX_RANKS; ++r) m.peer_delta[r] = c->peer_delta[r];
  m.xkey = c->xkey;
  c->mega_dirty = false;
  return F5_OK;
}

// engine of the next step (auto: persistent when it fits, else the graph)
static int resolve_engine(f5_ctx *c, int &eng) {
  if (c->engine == F5_ENGINE_GRAPH) {
    eng = F5_ENGINE_GRAPH;
    return build_graph(c);
  }
  bool unsupported = false;
  int rc = build_mega(c, unsupported);
  if (rc == F5_OK) {
    eng = F5_ENGINE_PERSISTENT;
    return F5_OK;
  }
  if (!unsupported || c->engine == F5_ENGINE_PERSISTENT) return rc;
  eng = F5_ENGINE_GRAPH;
  return build_graph(c);
}

static int launch_step(f5_ctx *c, int eng) {
  if (eng == F5_ENGINE_PERSISTENT)
    return cuda_status(launch_mega(c->margs, c->mega_grid, c->mega_smem, c->st), "persistent decode step");
  return cuda_status(cudaGraphLaunch(c->step_exec, c->st), "decode step");
}

static int finish_host(f5_ctx *c, const char *what) {
  F5_CU(cudaMemcpyAsync(c->h_params, c->params, sizeof(StepParams), cudaMemcpyDeviceToHost, c->st), what);
  F5_CU(cudaStreamSynchronize(c->st), what);
  if (c->h_params->err & DERR_Y32_OVERFLOW) return set_error(F5_EOVERFLOW, "%s: y32 overflow (ref/w4a8_ref.py:288)", what);
  if (c->h_params->err & DERR_TIMEOUT) {
    // an aborted persistent step may leave tagged words half written
    if (c->twin_mem) cudaMemsetAsync(c->twin_mem, 0, c->twin_bytes, c->st);
    return set_error(F5_ETIMEOUT, "%s: a bounded device wait gave up", what);
  }
  if (c->h_params->err & DERR_KV_FULL) return set_error(F5_ESTATE, "%s: KV cache full or position outside the RoPE table", what);
  if (c->h_params->err & DERR_RANGE) return set_error(F5_EINVAL, "%s: token id outside the vocabulary", what);
  return F5_OK;
}

}  // namespace f5

using namespace f5;

extern "C" {

int f5_ctx_create(const f5_config *cfg, int device, f5_ctx **out) {
  if (!cfg || !out) return set_error(F5_EINVAL, "f5_ctx_create: null argument");
  if (cfg->abi_version != F5_ABI_VERSION) return set_error(F5_EINVAL, "ABI version %d != %d", cfg->abi_version, F5_ABI_VERSION);
  if (cfg->n_layers <= 0 || cfg->vocab <= 0 || cfg->max_T <= 0 || cfg->world_size < 1 || cfg->rank < 0 ||
      cfg->rank >= cfg->world_size || (cfg->norm_mode != 0 && cfg->norm_mode != 1))
    return set_error(F5_EINVAL, "f5_ctx_create: bad config");
  if (!cfg->layer_types || (int)strlen(cfg->layer_types) != cfg->n_layers)
    return set_error(F5_EINVAL, "layer_types must hold n_layers chars of 'D' / 'A'");
  if (cfg->max_T > 6144) return set_error(F5_EINVAL, "max_T=%d above the 6144-token KV capacity of a context", cfg->max_T);
  DevGuard dg(device);
  f5_ctx *c = new f5_ctx();
  c->cfg = *cfg;
  c->cfg.max_T = (cfg->max_T + 15) & ~15;   // KV rows are bulk-copied in 16-row multiples
  c->device = device;
  std::string types(cfg->layer_types);
  c->cfg.layer_types = nullptr;
  int rc = F5_OK;
  auto fail = [&](int r) { f5_ctx_destroy(c); return r; };
  if ((rc = cuda_status(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking), "stream"))) return fail(rc);
  c->L.resize(cfg->n_layers);
  for (int i = 0; i < cfg->n_layers; ++i) {
    Layer &l = c->L[i];
    if (types[i] != 'A' && types[i] != 'D') return fail(set_error(F5_EINVAL, "layer_types[%d] = '%c'", i, types[i]));
    l.attn = types[i] == 'A';
    if ((rc = alloc(c, (void **)&l.ln1, H * 4)) || (rc = alloc(c, (void **)&l.ln2, H * 4))) return fail(rc);
    if (l.attn) {
      const size_t kv = (size_t)NKV * cfg->max_T;
      if ((rc = alloc(c, (void **)&l.q_norm, HD * 4)) || (rc = alloc(c, (void **)&l.k_norm, HD * 4)) ||
          (rc = alloc(c, (void **)&l.k8, kv * HD)) || (rc = alloc(c, (void **)&l.v8, kv * HD)) ||
          (rc = alloc(c, (void **)&l.ke, kv)) || (rc = alloc(c, (void **)&l.ve, kv)) ||
          (rc = alloc(c, (void **)&l.ka, 16)))
        return fail(rc);
    } else {
      if ((rc = alloc(c, (void **)&l.conv_w, (size_t)CONV_DIM * 4 * 4)) || (rc = alloc(c, (void **)&l.dt_bias, LNH * 4)) ||
          (rc = alloc(c, (void **)&l.A, LNH * 4)) || (rc = alloc(c, (void **)&l.norm_w, LDV * 4)) ||
          (rc = alloc(c, (void **)&l.conv, (size_t)CONV_DIM * 4 * 2)) ||
          (rc = alloc(c, (void **)&l.S, (size_t)LNH * LDK * LDV * 2)) || (rc = alloc(c, (void **)&l.kh, LNH * 4)))
        return fail(rc);
    }
  }
  if ((rc = alloc(c, (void **)&c->ln_f, H * 4)) || (rc = alloc(c, (void **)&c->x16, H * 2)) ||
      (rc = alloc(c, (void **)&c->qkv16, CONV_DIM * 2)) || (rc = alloc(c, (void **)&c->z16, LVD * 2)) ||
      (rc = alloc(c, (void **)&c->b16, 64 * 2)) || (rc = alloc(c, (void **)&c->a16, 64 * 2)) ||
      (rc = alloc(c, (void **)&c->on16, LVD * 2)) || (rc = alloc(c, (void **)&c->qg16, NQ * HD * 2 * 2)) ||
      (rc = alloc(c, (void **)&c->k16, NKV * HD * 2)) || (rc = alloc(c, (void **)&c->v16, NKV * HD * 2)) ||
      (rc = alloc(c, (void **)&c->prod16, FFN * 2)) || (rc = alloc(c, (void **)&c->prod64, NQ * HD * 8)) ||
      (rc = alloc(c, (void **)&c->x8, FFN)) || (rc = alloc(c, (void **)&c->xmeta, 16)) ||
      (rc = alloc(c, (void **)&c->qkvc16, CONV_DIM * 2)) || (rc = alloc(c, (void **)&c->gates, 2 * LNH * 4)) ||
      (rc = alloc(c, (void **)&c->key, 8)) || (rc = alloc(c, (void **)&c->stats, 4 * 8)) ||
      (rc = alloc(c, (void **)&c->err, 4)) || (rc = alloc(c, (void **)&c->params, sizeof(StepParams))))
    return fail(rc);
  if ((rc = cuda_status(cudaMallocHost(&c->h_params, sizeof(StepParams)), "cudaMallocHost"))) return fail(rc);
  memset(c->h_params, 0, sizeof(StepParams));
  if ((rc = cuda_status(cudaStreamSynchronize(c->st), "create sync"))) return fail(rc);
  *out = c;
  return F5_OK;
}

int f5_ctx_destroy(f5_ctx *c) {
  if (!c) return F5_OK;
  DevGuard dg(c->device);
  if (c->st) cudaStreamSynchronize(c->st);
  if (c->step_exec) cudaGraphExecDestroy(c->step_exec);
  free_mega(c);
  for (int r = 0; r < F5_MAX_RANKS; ++r)
    if (c->peer_base[r]) cudaIpcCloseMemHandle(c->peer_base[r]);
  for (void *p : c->allocs) cudaFree(p);
  if (c->h_params) cudaFreeHost(c->h_params);
  if (c->st) cudaStreamDestroy(c->st);
  delete c;
  return F5_OK;
}

int f5_ctx_upload_matrix(f5_ctx *c, int layer, int slot, const uint8_t *img, int N, int K, int g, int e, int sh) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!img) return set_error(F5_EINVAL, "f5_ctx_upload_matrix: null image");
  DevGuard dg(c->device);
  DevMat *m;
  if ((rc = prep_matrix(c, layer, slot, N, K, g, e, sh, m))) return rc;
  F5_CU(cudaMemcpyAsync(m->w, img + (size_t)m->row0 * m->stride, (size_t)m->rows * m->stride,
                        cudaMemcpyHostToDevice, c->st), "upload matrix");
  F5_CU(cudaStreamSynchronize(c->st), "upload matrix");
  return F5_OK;
}

int f5_ctx_synth_matrix(f5_ctx *c, int layer, int slot, int N, int K, int g, int e, int sh, uint64_t key_w,
                        uint64_t key_m, int symmetric) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  DevMat *m;
  if ((rc = prep_matrix(c, layer, slot, N, K, g, e, sh, m))) return rc;
  F5_CU(launch_synth_w4(m->w, m->rows, K, g, m->row0, key_w, key_m, symmetric, c->st), "synth matrix");
  return F5_OK;
}

int f5_ctx_upload_vector(f5_ctx *c, int layer, int kind, const int64_t *v, int n) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!v) return set_error(F5_EINVAL, "f5_ctx_upload_vector: null data");
  DevGuard dg(c->device);
  int32_t *dst = nullptr;
  int want = 0;
  if (layer == -1) {
    if (kind == F5_VEC_LN_F) { dst = c->ln_f; want = H; }
  } else if (layer >= 0 && layer < (int)c->L.size()) {
    Layer &l = c->L[layer];
    switch (kind) {
      case F5_VEC_LN1: dst = l.ln1; want = H; break;
      case F5_VEC_LN2: dst = l.ln2; want = H; break;
      case F5_VEC_Q_NORM: dst = l.q_norm; want = HD; break;
      case F5_VEC_K_NORM: dst = l.k_norm; want = HD; break;
      case F5_VEC_CONV_W: dst = l.conv_w; want = CONV_DIM * 4; break;
      case F5_VEC_DT_BIAS: dst = l.dt_bias; want = LNH; break;
      case F5_VEC_A: dst = l.A; want = LNH; break;
      case F5_VEC_NORM_W: dst = l.norm_w; want = LDV; break;
      default: break;
    }
  }
  if (!dst) return set_error(F5_EINVAL, "no vector kind %d in layer %d", kind, layer);
  if (n != want) return set_error(F5_EINVAL, "vector kind %d: %d values, expected %d", kind, n, want);
  std::vector<int32_t> tmp(n);
  for (int i = 0; i < n; ++i) {
    if (v[i] < INT32_MIN || v[i] > INT32_MAX) return set_error(F5_EINVAL, "vector kind %d: value outside int32", kind);
    tmp[i] = (int32_t)v[i];
  }
  F5_CU(cudaMemcpyAsync(dst, tmp.data(), n * 4, cudaMemcpyHostToDevice, c->st), "upload vector");
  F5_CU(cudaStreamSynchronize(c->st), "upload vector");
  return F5_OK;
}

static int ensure_emb(f5_ctx *c) {
  if (!c->emb) {
    F5_ALLOC(c, c->emb, (size_t)c->cfg.vocab * H * 2);
    c->graph_dirty = c->mega_dirty = true;
  }
  return F5_OK;
}

int f5_ctx_upload_embedding(f5_ctx *c, const int16_t *emb, int vocab, int h) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!emb || vocab != c->cfg.vocab || h != H) return set_error(F5_EINVAL, "embedding must be [vocab][4096] int16");
  DevGuard dg(c->device);
  if ((rc = ensure_emb(c))) return rc;
  F5_CU(cudaMemcpyAsync(c->emb, emb, (size_t)vocab * H * 2, cudaMemcpyHostToDevice, c->st), "upload embedding");
  F5_CU(cudaStreamSynchronize(c->st), "upload embedding");
  return F5_OK;
}

int f5_ctx_synth_embedding(f5_ctx *c, uint64_t key_e) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  if ((rc = ensure_emb(c))) return rc;
  F5_CU(launch_synth_emb(c->emb, c->cfg.vocab, H, 0, key_e, c->st), "synth embedding");
  return F5_OK;
}

int f5_ctx_upload_rope(f5_ctx *c, const int16_t *tab, int npos) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!tab || npos <= 0) return set_error(F5_EINVAL, "RoPE table must be [npos][128] int16");
  DevGuard dg(c->device);
  if (c->rope && npos > c->rope_npos) return set_error(F5_EINVAL, "RoPE table cannot grow");
  if (!c->rope) F5_ALLOC(c, c->rope, (size_t)npos * 128 * 2);
  c->rope_npos = npos;
  F5_CU(cudaMemcpyAsync(c->rope, tab, (size_t)npos * 128 * 2, cudaMemcpyHostToDevice, c->st), "upload rope");
  F5_CU(cudaStreamSynchronize(c->st), "upload rope");
  c->graph_dirty = c->mega_dirty = true;
  return F5_OK;
}

int f5_ctx_reset(f5_ctx *c) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  for (Layer &l : c->L) {
    if (l.attn) {
      const size_t kv = (size_t)NKV * c->cfg.max_T;
      F5_CU(cudaMemsetAsync(l.k8, 0, kv * HD, c->st), "reset");
      F5_CU(cudaMemsetAsync(l.v8, 0, kv * HD, c->st), "reset");
      F5_CU(cudaMemsetAsync(l.ke, 0, kv, c->st), "reset");
      F5_CU(cudaMemsetAsync(l.ve, 0, kv, c->st), "reset");
    } else {
      F5_CU(cudaMemsetAsync(l.conv, 0, (size_t)CONV_DIM * 4 * 2, c->st), "reset");
      F5_CU(cudaMemsetAsync(l.S, 0, (size_t)LNH * LDK * LDV * 2, c->st), "reset");
    }
  }
  F5_CU(cudaMemsetAsync(c->params, 0, sizeof(StepParams), c->st), "reset");
  if (c->twin_mem) F5_CU(cudaMemsetAsync(c->twin_mem, 0, c->twin_bytes, c->st), "reset");
  F5_CU(cudaMemsetAsync(c->err, 0, 4, c->st), "reset");
  F5_CU(cudaMemsetAsync(c->stats, 0, 4 * 8, c->st), "reset");
  F5_CU(cudaStreamSynchronize(c->st), "reset");
  return F5_OK;
}

int f5_ctx_set_position(f5_ctx *c, int T, int pos) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (T < 0 || T > c->cfg.max_T) return set_error(F5_EINVAL, "T=%d outside [0, max_T]", T);
  DevGuard dg(c->device);
  F5_CU(cudaMemcpyAsync(c->h_params, c->params, sizeof(StepParams), cudaMemcpyDeviceToHost, c->st), "set position");
  F5_CU(cudaStreamSynchronize(c->st), "set position");
  c->h_params->T = T;
  c->h_params->pos = pos;
  F5_CU(cudaMemcpyAsync(c->params, c->h_params, sizeof(StepParams), cudaMemcpyHostToDevice, c->st), "set position");
  F5_CU(cudaStreamSynchronize(c->st), "set position");
  return F5_OK;
}

int f5_ctx_get_position(f5_ctx *c, int *T, int *pos) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  F5_CU(cudaMemcpyAsync(c->h_params, c->params, sizeof(StepParams), cudaMemcpyDeviceToHost, c->st), "get position");
  F5_CU(cudaStreamSynchronize(c->st), "get position");
  if (T) *T = c->h_params->T;
  if (pos) *pos = c->h_params->pos;
  return F5_OK;
}

int f5_ctx_set_logits(f5_ctx *c, int on) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  if (on && !c->logits) F5_ALLOC(c, c->logits, (size_t)c->cfg.vocab * 4);
  if ((bool)on != c->want_logits) {
    c->want_logits = on != 0;
    c->graph_dirty = c->mega_dirty = true;
  }
  return F5_OK;
}

int f5_ctx_topk(f5_ctx *c, f5_topk32 *out) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!out) return set_error(F5_EINVAL, "f5_ctx_topk: null out");
  if (!c->logits || !c->want_logits)
    return set_error(F5_ESTATE, "f5_ctx_topk: logits not stored (f5_ctx_set_logits(ctx, 1) before the step)");
  if (c->cfg.world_size > 1) return set_error(F5_ESTATE, "f5_ctx_topk: single-GPU contexts only");
  if (!c->ln_f) return set_error(F5_ESTATE, "f5_ctx_topk: final norm not uploaded");
  DevGuard dg(c->device);
  const int vocab = c->cfg.vocab;
  if (!c->tk_ws) {
    F5_ALLOC(c, c->tk_ws, f5::topk32_ws_bytes(vocab));
    F5_ALLOC(c, c->tk_out, sizeof(f5_topk32));
    F5_ALLOC(c, c->tk_xt, (size_t)(H / 128) * 16 * 128);
    F5_ALLOC(c, c->tk_xmeta, 16 * 2 * sizeof(int));
  }
  // e_x: the head's prologue (rmsnorm_fx(x, ln_f, RS_F, one_plus=0) then
  // DYNQ8, ref/fidelity_check.py:442-446) over the final residual
  f5::BprepArgs pa = {};
  pa.pro.mode = PRO_RMSNORM;
  pa.pro.src = c->x16;
  pa.pro.w = c->ln_f;
  pa.pro.in_f = RS_F;
  pa.pro.one_plus = 0;
  pa.K = H;
  pa.NG = H / 128;
  pa.B = 1;
  pa.Bp = 16;
  pa.xmeta = c->tk_xmeta;
  pa.xt = c->tk_xt;
  pa.err = c->err;
  F5_CU(f5::launch_bprep(pa, c->st, false), "f5_ctx_topk prologue");
  F5_CU(f5::launch_topk32(c->logits, vocab, c->tk_ws, c->tk_out, c->tk_xmeta, c->st), "f5_ctx_topk");
  F5_CU(cudaMemcpyAsync(out, c->tk_out, sizeof(f5_topk32), cudaMemcpyDeviceToHost, c->st), "f5_ctx_topk");
  F5_CU(cudaStreamSynchronize(c->st), "f5_ctx_topk");
  return F5_OK;
}

int f5_ctx_stream(f5_ctx *c, void **stream) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!stream) return set_error(F5_EINVAL, "f5_ctx_stream: null out");
  *stream = (void *)c->st;
  return F5_OK;
}

int f5_ctx_prepare(f5_ctx *c) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  int eng;
  return resolve_engine(c, eng);
}

int f5_ctx_set_engine(f5_ctx *c, int engine) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (engine != F5_ENGINE_GRAPH && engine != F5_ENGINE_PERSISTENT)
    return set_error(F5_EINVAL, "f5_ctx_set_engine: engine %d", engine);
  c->engine = engine;
  return F5_OK;
}

int f5_ctx_get_engine(f5_ctx *c, int *engine) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!engine) return set_error(F5_EINVAL, "f5_ctx_get_engine: null out");
  DevGuard dg(c->device);
  return resolve_engine(c, *engine);
}

int f5_ctx_ipc_handle(f5_ctx *c, void *handle, size_t cap) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!handle || cap < sizeof(cudaIpcMemHandle_t)) return set_error(F5_EINVAL, "f5_ctx_ipc_handle: %zu-byte buffer", sizeof(cudaIpcMemHandle_t));
  DevGuard dg(c->device);
  if ((rc = ensure_twins(c))) return rc;
  cudaIpcMemHandle_t h;
  F5_CU(cudaIpcGetMemHandle(&h, c->twin_mem), "cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof(h));
  return F5_OK;
}

int f5_ctx_attach_peers(f5_ctx *c, const void *handles, int n) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!handles || n != c->cfg.world_size || n > F5_MAX_RANKS)
    return set_error(F5_EINVAL, "f5_ctx_attach_peers: %d handles for world size %d", n, c->cfg.world_size);
  if (c->peers_attached) return set_error(F5_ESTATE, "peers already attached");
  DevGuard dg(c->device);
  if ((rc = ensure_twins(c))) return rc;
  const cudaIpcMemHandle_t *hs = static_cast<const cudaIpcMemHandle_t *>(handles);
  for (int r = 0; r < n; ++r) {
    if (r == c->cfg.rank) {
      c->peer_delta[r] = 0;
      continue;
    }
    void *p = nullptr;
    F5_CU(cudaIpcOpenMemHandle(&p, hs[r], cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    c->peer_base[r] = p;
    c->peer_delta[r] = static_cast<char *>(p) - reinterpret_cast<char *>(c->twin_mem);
  }
  c->peers_attached = true;
  c->graph_dirty = c->mega_dirty = true;
  return F5_OK;
}

int f5_ctx_trace_step(f5_ctx *c, uint64_t *out, size_t cap, int *grid, int *nops) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  bool unsupported = false;
  if ((rc = build_mega(c, unsupported))) return rc;
  if (grid) *grid = c->mega_grid;
  if (nops) *nops = c->margs.nops;
  if (!out) return F5_OK;
  const size_t n = (size_t)c->mega_grid * c->margs.nops * MEGA_TRACE_SLOTS;
  if (cap < n) return set_error(F5_EINVAL, "f5_ctx_trace_step: %zu slots, need %zu", cap, n);
  unsigned long long *d = nullptr;
  F5_CU(cudaMalloc(&d, n * 8), "trace buffer");
  MegaArgs m = c->margs;
  m.trace = d;
  cudaError_t e = cudaMemsetAsync(d, 0, n * 8, c->st);
  if (e == cudaSuccess) e = launch_mega_traced(m, c->mega_grid, c->mega_smem, c->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, d, n * 8, cudaMemcpyDeviceToHost, c->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->st);
  cudaFree(d);
  F5_CU(e, "f5_ctx_trace_step");
  return finish_host(c, "f5_ctx_trace_step");
}

int f5_decode_step(f5_ctx *c, int32_t tok, int32_t pos, int32_t *next_tok, int32_t *max_logit) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  int eng;
  if ((rc = resolve_engine(c, eng))) return rc;
  // Only the step's inputs travel: tok and pos, the first two words of the
  // parameter block, from the pinned host copy (no read-back of the block
  // first: T and the launch counter stay the device's own words); then the
  // error words are cleared.  finish_host's read-back rewrites the host copy
  // after the step, on the same stream.
  static_assert(offsetof(StepParams, tok) == 0 && offsetof(StepParams, pos) == sizeof(int32_t), "tok, pos first");
  c->h_params->tok = tok;
  c->h_params->pos = pos;
  F5_CU(cudaMemcpyAsync(c->params, c->h_params, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, c->st), "decode step");
  F5_CU(cudaMemsetAsync(&c->params->err, 0, sizeof(uint32_t), c->st), "decode step");
  F5_CU(cudaMemsetAsync(c->err, 0, 4, c->st), "decode step");
  if ((rc = launch_step(c, eng))) return rc;
  if ((rc = finish_host(c, "f5_decode_step"))) return rc;
  if (next_tok) *next_tok = c->h_params->next_tok;
  if (max_logit) *max_logit = c->h_params->max_val;
  return F5_OK;
}

int f5_decode_launch(f5_ctx *c, int n_steps, void *stream_unused) {
  (void)stream_unused;
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  int eng;
  if ((rc = resolve_engine(c, eng))) return rc;
  for (int i = 0; i < n_steps; ++i)
    if ((rc = launch_step(c, eng))) return rc;
  return F5_OK;
}

int f5_decode_prefill(f5_ctx *c, const int32_t *tokens, int n) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (n < 0 || (n > 0 && !tokens)) return set_error(F5_EINVAL, "f5_decode_prefill: n=%d, tokens %p", n, tokens);
  if (n > c->cfg.max_T) return set_error(F5_EINVAL, "f5_decode_prefill: %d tokens, KV capacity %d", n, c->cfg.max_T);
  DevGuard dg(c->device);
  int eng;
  if ((rc = resolve_engine(c, eng))) return rc;
  if (!c->prompt) F5_ALLOC(c, c->prompt, (size_t)c->cfg.max_T * sizeof(int32_t));
  F5_CU(cudaMemcpyAsync(c->prompt, tokens, (size_t)n * sizeof(int32_t), cudaMemcpyHostToDevice, c->st),
        "f5_decode_prefill");
  for (int i = 0; i < n; ++i) {
    k_set_token<<<1, 1, 0, c->st>>>(c->params, c->prompt, i);
    F5_CU(cudaGetLastError(), "f5_decode_prefill");
    if ((rc = launch_step(c, eng))) return rc;
  }
  return F5_OK;
}

int f5_ctx_sync(f5_ctx *c, int32_t *last_tok, int32_t *max_logit) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DevGuard dg(c->device);
  if ((rc = finish_host(c, "f5_ctx_sync"))) return rc;
  if (last_tok) *last_tok = c->h_params->next_tok;
  if (max_logit) *max_logit = c->h_params->max_val;
  return F5_OK;
}

int f5_ctx_time_step(f5_ctx *c, int reps, double *out, int nout) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!out || nout < 8 || reps < 1) return set_error(F5_EINVAL, "f5_ctx_time_step: out[8] and reps >= 1 required");
  DevGuard dg(c->device);
  if ((rc = ready(c))) return rc;
  for (int i = 0; i < 8; ++i) out[i] = 0;
  for (int r = 0; r < reps; ++r) {
    c->timing = true;
    c->timed.clear();
    cudaError_t e = enqueue_step(c, false);
    c->timing = false;
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->st);
    for (auto &t : c->timed) {
      float ms = 0;
      if (e == cudaSuccess) cudaEventElapsedTime(&ms, t.a, t.b);
      const int slot = t.kind == TK_GEMV ? 0 : (t.kind == TK_DN ? 3 : (t.kind == TK_ATTN ? 4 : 5));
      out[slot] += ms;
      if (t.kind == TK_GEMV) { out[1] += t.bytes; out[2] += 1; }
      out[6] += ms;
      out[7] += 1;
      cudaEventDestroy(t.a);
      cudaEventDestroy(t.b);
    }
    c->timed.clear();
    if (e != cudaSuccess) return cuda_status(e, "f5_ctx_time_step");
  }
  for (int i = 0; i < 8; ++i) out[i] /= reps;
  return finish_host(c, "f5_ctx_time_step");
}

int f5_layer_step(f5_ctx *c, int layer, int16_t *x16_inout, int T, int pos) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!x16_inout || layer < 0 || layer >= (int)c->L.size()) return set_error(F5_EINVAL, "f5_layer_step: bad layer / buffer");
  DevGuard dg(c->device);
  if ((rc = layer_ready(c, layer))) return rc;
  F5_CU(cudaMemcpyAsync(c->h_params, c->params, sizeof(StepParams), cudaMemcpyDeviceToHost, c->st), "layer step");
  F5_CU(cudaStreamSynchronize(c->st), "layer step");
  if (T < 0 || T >= c->cfg.max_T) return set_error(F5_ESTATE, "f5_layer_step: T=%d outside [0, max_T)", T);
  c->h_params->T = T;
  c->h_params->pos = pos;
  c->h_params->err = 0;
  F5_CU(cudaMemcpyAsync(c->params, c->h_params, sizeof(StepParams), cudaMemcpyHostToDevice, c->st), "layer step");
  F5_CU(cudaMemsetAsync(c->err, 0, 4, c->st), "layer step");
  F5_CU(cudaMemcpyAsync(c->x16, x16_inout, H * 2, cudaMemcpyHostToDevice, c->st), "layer step");
  F5_CU(enqueue_layer(c, layer, false), "layer step");
  {
    StepParams *p = c->params;
    const uint32_t *er = c->err;
    void *args[] = {&p, &er};
    F5_CU(launch_pdl((const void *)k_collect_err, args, dim3(1), dim3(1), c->st, false), "layer step");
  }
  F5_CU(cudaMemcpyAsync(x16_inout, c->x16, H * 2, cudaMemcpyDeviceToHost, c->st), "layer step");
  return finish_host(c, "f5_layer_step");
}

int f5_ctx_read(f5_ctx *c, int what, int layer, void *dst, size_t bytes) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!dst) return set_error(F5_EINVAL, "f5_ctx_read: null destination");
  DevGuard dg(c->device);
  const void *src = nullptr;
  size_t n = 0;
  Layer *l = (layer >= 0 && layer < (int)c->L.size()) ? &c->L[layer] : nullptr;
  switch (what) {
    case F5_BUF_X16: src = c->x16; n = H * 2; break;
    case F5_BUF_QKV16: src = c->qkv16; n = CONV_DIM * 2; break;
    case F5_BUF_Z16: src = c->z16; n = LVD * 2; break;
    case F5_BUF_B16: src = c->b16; n = LNH * 2; break;
    case F5_BUF_A16: src = c->a16; n = LNH * 2; break;
    case F5_BUF_ON16: src = c->on16; n = LVD * 2; break;
    case F5_BUF_QG16: src = c->qg16; n = NQ * HD * 2 * 2; break;
    case F5_BUF_K16: src = c->k16; n = NKV * HD * 2; break;
    case F5_BUF_V16: src = c->v16; n = NKV * HD * 2; break;
    case F5_BUF_PROD64: src = c->prod64; n = NQ * HD * 8; break;
    case F5_BUF_PROD16: src = c->prod16; n = FFN * 2; break;
    case F5_BUF_STATS: src = c->stats; n = 4 * 8; break;
    case F5_BUF_DN_S: if (l && !l->attn) { src = l->S; n = (size_t)LNH * LDK * LDV * 2; } break;
    case F5_BUF_DN_CONV: if (l && !l->attn) { src = l->conv; n = (size_t)CONV_DIM * 4 * 2; } break;
    case F5_BUF_DN_KH: if (l && !l->attn) { src = l->kh; n = LNH * 4; } break;
    case F5_BUF_K8: if (l && l->attn) { src = l->k8; n = (size_t)NKV * c->cfg.max_T * HD; } break;
    case F5_BUF_KE: if (l && l->attn) { src = l->ke; n = (size_t)NKV * c->cfg.max_T; } break;
    case F5_BUF_V8: if (l && l->attn) { src = l->v8; n = (size_t)NKV * c->cfg.max_T * HD; } break;
    case F5_BUF_VE: if (l && l->attn) { src = l->ve; n = (size_t)NKV * c->cfg.max_T; } break;
    case F5_BUF_KA: if (l && l->attn) { src = l->ka; n = 4; } break;
    case F5_BUF_LOGITS: if (c->logits) { src = c->logits; n = (size_t)c->cfg.vocab * 4; } break;
    case F5_BUF_QKVC16: src = c->qkvc16; n = CONV_DIM * 2; break;
    case F5_BUF_GATES: src = c->gates; n = 2 * LNH * 4; break;
    default: break;
  }
  if (!src) return set_error(F5_EINVAL, "f5_ctx_read: no buffer %d for layer %d", what, layer);
  if (bytes != n) return set_error(F5_EINVAL, "f5_ctx_read: buffer %d holds %zu bytes, asked %zu", what, n, bytes);
  F5_CU(cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, c->st), "f5_ctx_read");
  F5_CU(cudaStreamSynchronize(c->st), "f5_ctx_read");
  return F5_OK;
}

int f5_ctx_write(f5_ctx *c, int what, int layer, const void *src, size_t bytes) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!src) return set_error(F5_EINVAL, "f5_ctx_write: null source");
  DevGuard dg(c->device);
  void *dst = nullptr;
  size_t n = 0;
  Layer *l = (layer >= 0 && layer < (int)c->L.size()) ? &c->L[layer] : nullptr;
  switch (what) {
    case F5_BUF_X16: dst = c->x16; n = H * 2; break;
    case F5_BUF_DN_S: if (l && !l->attn) { dst = l->S; n = (size_t)LNH * LDK * LDV * 2; } break;
    case F5_BUF_DN_CONV: if (l && !l->attn) { dst = l->conv; n = (size_t)CONV_DIM * 4 * 2; } break;
    case F5_BUF_K8: if (l && l->attn) { dst = l->k8; n = (size_t)NKV * c->cfg.max_T * HD; } break;
    case F5_BUF_KE: if (l && l->attn) { dst = l->ke; n = (size_t)NKV * c->cfg.max_T; } break;
    case F5_BUF_V8: if (l && l->attn) { dst = l->v8; n = (size_t)NKV * c->cfg.max_T * HD; } break;
    case F5_BUF_VE: if (l && l->attn) { dst = l->ve; n = (size_t)NKV * c->cfg.max_T; } break;
    default: break;
  }
  if (!dst) return set_error(F5_EINVAL, "f5_ctx_write: buffer %d of layer %d is not writable", what, layer);
  if (bytes != n) return set_error(F5_EINVAL, "f5_ctx_write: buffer %d holds %zu bytes, got %zu", what, n, bytes);
  F5_CU(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, c->st), "f5_ctx_write");
  F5_CU(cudaStreamSynchronize(c->st), "f5_ctx_write");
  return F5_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Reference-layout state images (ref/layer_fixed.py:1654-1666 new_cache_fx,
// the caches the reference's layer_decode_fx mutates).  DeltaNet layer:
// S int16 [LNH][LDK][LDV] then the conv window int64 [CONV_DIM][3], oldest
// first; attention layer at T tokens: k8 int8 [T][NKV][HD], ke int8
// [T][NKV], v8 int8 [T][NKV][HD], ve int8 [T][NKV] -- the reference's
// cache["k"][t][h] = (k8, ke) lists flattened in that order.
// ---------------------------------------------------------------------------
namespace {
size_t state_bytes_of(const f5_ctx *c, int layer, int T) {
  if (layer < 0 || layer >= (int)c->L.size() || T < 0) return 0;
  if (!c->L[layer].attn) return (size_t)LNH * LDK * LDV * 2 + (size_t)CONV_DIM * 3 * 8;
  return (size_t)T * NKV * (HD + 1) * 2;
}
}  // namespace

size_t f5_state_bytes(f5_ctx *c, int layer, int T) {
  if (!c) return 0;
  return state_bytes_of(c, layer, T);
}

int f5_state_save(f5_ctx *c, int layer, void *dst, size_t bytes) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!dst) return set_error(F5_EINVAL, "f5_state_save: null destination");
  if (layer < 0 || layer >= (int)c->L.size()) return set_error(F5_EINVAL, "f5_state_save: layer %d", layer);
  DevGuard dg(c->device);
  F5_CU(cudaMemcpyAsync(c->h_params, c->params, sizeof(StepParams), cudaMemcpyDeviceToHost, c->st), "f5_state_save");
  F5_CU(cudaStreamSynchronize(c->st), "f5_state_save");
  const int T = c->h_params->T;
  const size_t need = state_bytes_of(c, layer, T);
  if (bytes != need) return set_error(F5_EINVAL, "f5_state_save: layer %d at T=%d needs %zu bytes, got %zu", layer, T, need, bytes);
  const Layer &l = c->L[layer];
  uint8_t *out = static_cast<uint8_t *>(dst);
  if (!l.attn) {
    std::vector<int16_t> S((size_t)LNH * LDK * LDV), ring((size_t)CONV_DIM * 4);
    F5_CU(cudaMemcpyAsync(S.data(), l.S, S.size() * 2, cudaMemcpyDeviceToHost, c->st), "f5_state_save");
    F5_CU(cudaMemcpyAsync(ring.data(), l.conv, ring.size() * 2, cudaMemcpyDeviceToHost, c->st), "f5_state_save");
    F5_CU(cudaStreamSynchronize(c->st), "f5_state_save");
    int16_t *so = reinterpret_cast<int16_t *>(out);
    // device [head][dv / 32][dk][dv % 32] -> reference [head][dk][dv]
    for (int h = 0; h < LNH; ++h)
      for (int q = 0; q < LDV / 32; ++q)
        for (int k = 0; k < LDK; ++k)
          for (int i = 0; i < 32; ++i)
            so[((size_t)h * LDK + k) * LDV + q * 32 + i] = S[(((size_t)h * (LDV / 32) + q) * LDK + k) * 32 + i];
    int64_t *co = reinterpret_cast<int64_t *>(out + (size_t)LNH * LDK * LDV * 2);
    // ring slot T % 4 takes this step's input; the other three, oldest first
    for (int ch = 0; ch < CONV_DIM; ++ch)
      for (int j = 0; j < 3; ++j) co[(size_t)ch * 3 + j] = ring[(size_t)ch * 4 + ((T - 3 + j) & 3)];
    return F5_OK;
  }
  const size_t mt = (size_t)c->cfg.max_T;
  std::vector<int8_t> k8(NKV * mt * HD), ke(NKV * mt), v8(NKV * mt * HD), ve(NKV * mt);
  F5_CU(cudaMemcpyAsync(k8.data(), l.k8, k8.size(), cudaMemcpyDeviceToHost, c->st), "f5_state_save");
  F5_CU(cudaMemcpyAsync(ke.data(), l.ke, ke.size(), cudaMemcpyDeviceToHost, c->st), "f5_state_save");
  F5_CU(cudaMemcpyAsync(v8.data(), l.v8, v8.size(), cudaMemcpyDeviceToHost, c->st), "f5_state_save");
  F5_CU(cudaMemcpyAsync(ve.data(), l.ve, ve.size(), cudaMemcpyDeviceToHost, c->st), "f5_state_save");
  F5_CU(cudaStreamSynchronize(c->st), "f5_state_save");
  int8_t *o = reinterpret_cast<int8_t *>(out);
  const size_t rows = (size_t)T * NKV;
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < NKV; ++h) {
      const size_t r = (size_t)t * NKV + h, dr = (size_t)h * mt + t;
      memcpy(o + r * HD, k8.data() + dr * HD, HD);
      o[rows * HD + r] = ke[dr];
      memcpy(o + rows * (HD + 1) + r * HD, v8.data() + dr * HD, HD);
      o[rows * (2 * HD + 1) + r] = ve[dr];
    }
  return F5_OK;
}

int f5_state_load(f5_ctx *c, int layer, const void *src, size_t bytes, int T) {
  int rc = check_ctx(c);
  if (rc) return rc;
  if (!src) return set_error(F5_EINVAL, "f5_state_load: null source");
  if (layer < 0 || layer >= (int)c->L.size()) return set_error(F5_EINVAL, "f5_state_load: layer %d", layer);
  if (T < 0 || T > c->cfg.max_T) return set_error(F5_EINVAL, "f5_state_load: T=%d outside [0, max_T]", T);
  const size_t need = state_bytes_of(c, layer, T);
  if (bytes != need) return set_error(F5_EINVAL, "f5_state_load: layer %d at T=%d needs %zu bytes, got %zu", layer, T, need, bytes);
  DevGuard dg(c->device);
  const Layer &l = c->L[layer];
  const uint8_t *in = static_cast<const uint8_t *>(src);
  if (!l.attn) {
    std::vector<int16_t> S((size_t)LNH * LDK * LDV), ring((size_t)CONV_DIM * 4, 0);
    const int16_t *si = reinterpret_cast<const int16_t *>(in);
    for (int h = 0; h < LNH; ++h)
      for (int q = 0; q < LDV / 32; ++q)
        for (int k = 0; k < LDK; ++k)
          for (int i = 0; i < 32; ++i)
            S[(((size_t)h * (LDV / 32) + q) * LDK + k) * 32 + i] = si[((size_t)h * LDK + k) * LDV + q * 32 + i];
    const int64_t *ci = reinterpret_cast<const int64_t *>(in + (size_t)LNH * LDK * LDV * 2);
    for (int ch = 0; ch < CONV_DIM; ++ch)
      for (int j = 0; j < 3; ++j) {
        const int64_t v = ci[(size_t)ch * 3 + j];
        if (v < -32768 || v > 32767)
          return set_error(F5_EINVAL, "f5_state_load: conv window value %lld of channel %d is not int16", (long long)v, ch);
        ring[(size_t)ch * 4 + ((T - 3 + j) & 3)] = (int16_t)v;
      }
    F5_CU(cudaMemcpyAsync(l.S, S.data(), S.size() * 2, cudaMemcpyHostToDevice, c->st), "f5_state_load");
    F5_CU(cudaMemcpyAsync(l.conv, ring.data(), ring.size() * 2, cudaMemcpyHostToDevice, c->st), "f5_state_load");
    F5_CU(cudaStreamSynchronize(c->st), "f5_state_load");
    return F5_OK;
  }
  const size_t mt = (size_t)c->cfg.max_T;
  std::vector<int8_t> k8(NKV * mt * HD, 0), ke(NKV * mt, 0), v8(NKV * mt * HD, 0), ve(NKV * mt, 0);
  const int8_t *i8 = reinterpret_cast<const int8_t *>(in);
  const size_t rows = (size_t)T * NKV;
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < NKV; ++h) {
      const size_t r = (size_t)t * NKV + h, dr = (size_t)h * mt + t;
      memcpy(k8.data() + dr * HD, i8 + r * HD, HD);
      ke[dr] = i8[rows * HD + r];
      memcpy(v8.data() + dr * HD, i8 + rows * (HD + 1) + r * HD, HD);
      ve[dr] = i8[rows * (2 * HD + 1) + r];
    }
  F5_CU(cudaMemcpyAsync(l.k8, k8.data(), k8.size(), cudaMemcpyHostToDevice, c->st), "f5_state_load");
  F5_CU(cudaMemcpyAsync(l.ke, ke.data(), ke.size(), cudaMemcpyHostToDevice, c->st), "f5_state_load");
  F5_CU(cudaMemcpyAsync(l.v8, v8.data(), v8.size(), cudaMemcpyHostToDevice, c->st), "f5_state_load");
  F5_CU(cudaMemcpyAsync(l.ve, ve.data(), ve.size(), cudaMemcpyHostToDevice, c->st), "f5_state_load");
  F5_CU(cudaStreamSynchronize(c->st), "f5_state_load");
  return F5_OK;
}
