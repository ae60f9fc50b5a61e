/*
 * f5b200 -- C ABI of the B200 (sm_100a) integer W4A8 decode path for
 * Qwen3.5-9B, a drop-in for the reference model's Python API
 * (coreyhahn/fable5_llm ref/w4a8_ref.py, ref/fixedpoint.py,
 * ref/layer_fixed.py and the seq_model decode step).
 *
 * The reference has no FFI of its own: its boundary is a Python API over
 * numpy arrays.  Each entry point below names the reference function it
 * replaces (file:line inside that project); the Python host package
 * fable5_llm_b200 binds these with ctypes and re-exposes the reference
 * names and signatures.
 *
 * Conventions
 *   - every function returns an int status: F5_OK (0) or a negative F5_E*;
 *     f5_last_error() returns the message of the calling thread's last error
 *     (the reference raises AssertionError / SystemExit instead);
 *   - `_dev` entry points take device pointers and a cudaStream_t passed as
 *     void* (NULL = legacy default stream) and do not synchronise;
 *   - `_host` entry points take host pointers, allocate device scratch per
 *     call, copy in, run, copy out and synchronise;
 *   - a context (f5_ctx) owns one GPU's model, state, stream and decode
 *     graph.  Calls on one context are not thread-safe; the caller
 *     serialises.
 */
#ifndef F5B200_H
#define F5B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define F5_ABI_VERSION 1

enum f5_status {
  F5_OK = 0,
  F5_EINVAL = -1,     /* bad argument (shape, range, null pointer)         */
  F5_ECUDA = -2,      /* CUDA runtime error                                 */
  F5_ENOMEM = -3,     /* device allocation failed                           */
  F5_ETIMEOUT = -4,   /* a bounded device wait gave up                      */
  F5_EOVERFLOW = -5,  /* a range assertion of the reference law failed      */
  F5_ESTATE = -6,     /* call out of order (missing upload, full KV cache)  */
  F5_ENCCL = -7       /* collective failed                                  */
};

/* GEMV epilogue modes (f5_gemv_seg.mode) */
enum f5_gemv_mode {
  F5_GM_Y32 = 0,      /* int32 y32 (ref/w4a8_ref.py:254-289)                    */
  F5_GM_TO16 = 1,     /* clip16(matvec_to)  (ref/layer_fixed.py:1224-1236)      */
  F5_GM_TO64 = 2,     /* int64 matvec_to                                        */
  F5_GM_RESID = 3,    /* out16 = clip16(out16 + clip16(matvec_to)) (:1675-1677) */
  F5_GM_SILU_MUL = 4, /* paired gate/up: clip16(rshr(silu(g)*u, 12)) (:1597-1604)*/
  F5_GM_ARGMAX = 5    /* running (max y32, lowest row) key (gen_model_script:641)*/
};

/* primitive ops of f5_prim_dev (each restates one ref/fixedpoint.py or
 * ref/layer_fixed.py function; see fable5_llm_b200/csrc/f5_int.cuh) */
enum f5_prim_op {
  F5_PR_RSHR = 0, F5_PR_SIGMOID = 1, F5_PR_SOFTPLUS = 2, F5_PR_SILU = 3,
  F5_PR_EXP_NEG = 4, F5_PR_RSQRT = 5, F5_PR_RECIP = 6, F5_PR_BF_SHIFT = 7,
  F5_PR_DYNQ8_E = 8, F5_PR_DN_NORM_SCALE = 9, F5_PR_EPS_NORM_SCALE = 10,
  F5_PR_EXP2_FRAC = 11
};

int f5_abi_version(void);
const char *f5_status_string(int status);
/* copy the calling thread's last error message into buf (always NUL-terminated) */
int f5_last_error(char *buf, size_t len);

/* ---------------------------------------------------------------------------
 * Stateless kernels on device pointers
 * ------------------------------------------------------------------------- */

/* One matrix segment of a fused GEMV launch.  All segments of a launch share
 * K, g, sh and the quantized input x8. */
typedef struct f5_gemv_seg {
  const uint8_t *w;   /* packed pack_ddr_rows image, row 0 (ref/w4a8_ref.py:349-370) */
  const uint8_t *w2;  /* F5_GM_SILU_MUL: the paired `up` image; else NULL        */
  void *out;          /* int32 / int16 / int64 output base, indexed by out_row0+row */
  int64_t *p_out;     /* optional int64 p = sum_g m_g*acc_g per row, or NULL     */
  int rows;
  int e, e2;          /* shared weight exponents (ref/w4a8_ref.py:168)           */
  int out_f, out_f2;  /* matvec_to output fraction bits                          */
  int mode;           /* enum f5_gemv_mode                                       */
  int out_row0;
} f5_gemv_seg;

/* Fused W4A8 GEMV + epilogue.  Replaces ref/w4a8_ref.py:254-289 matvec_y32
 * (and ref/seq_model.py:431-452 DDRWeights.matvec on packed images) plus the
 * ref/layer_fixed.py:1224-1236 matvec_to shift.  d_xmeta = {e_x, in_f} from
 * a DYNQ8 producer (NULL: 0, 0).  d_argmax must be zeroed by the caller
 * before an F5_GM_ARGMAX launch; d_err is an optional uint32 error word
 * (bit 0: |y32| >= 2^31).  max_blocks <= 0 picks 2 per SM. */
int f5_gemv_dev(const f5_gemv_seg *segs, int nseg, int K, int g, int sh,
                const int8_t *d_x8, const int *d_xmeta,
                unsigned long long *d_argmax, uint32_t *d_err,
                int max_blocks, int pdl, void *stream);

/* RMSNorm + DYNQ8 of one vector: ref/layer_fixed.py:1242-1278 rmsnorm_fx
 * followed by ref/fixedpoint.py:24-33 dyn_quant_i8.  n power of two <= 4096;
 * d_w int32 gains (Q14, one_plus adds 2^14).  d_xn (int16, nullable) gets the
 * normalised vector, d_x8 / d_meta = {e_x, in_f} its DYNQ8. */
int f5_rmsnorm_dynq8_dev(const int16_t *d_x16, const int32_t *d_w, int n, int in_f,
                         int one_plus, int16_t *d_xn, int8_t *d_x8, int *d_meta,
                         void *stream);

/* DYNQ8 (ref/fixedpoint.py:24-33) of an int16 vector, n <= 12288. */
int f5_dynq8_dev(const int16_t *d_x16, int n, int in_f, int8_t *d_x8, int *d_meta,
                 void *stream);

/* Element-wise integer primitive (enum f5_prim_op) over n int64 inputs;
 * d_in2 (nullable) is a per-element second argument (shift, P, k); arg0 is
 * the scalar form.  d_out2 (nullable) receives the exponent of RSQRT/RECIP. */
int f5_prim_dev(int op, const int64_t *d_in, const int64_t *d_in2, int64_t *d_out,
                int64_t *d_out2, int n, int arg0, int arg1, void *stream);

/* Seeded synthetic W4 image rows [row0, row0+nrows) written into d_img
 * (bench/test input generator; identical bytes to fable5_llm_b200/synth.py). */
int f5_synth_w4_dev(uint8_t *d_img, long long nrows, int K, int g, long long row0,
                    uint64_t key_w, uint64_t key_m, int symmetric, void *stream);
int f5_synth_emb_dev(int16_t *d_emb, long long nrows, int H, long long row0,
                     uint64_t key_e, void *stream);

/* Checkpoint quantization of one float matrix d_w [N][K] (device; float32,
 * or float64 when w_f64 is nonzero) into
 * the W4 row format, on the GPU, bit-identical to the reference's host
 * quantizers (g = 128):
 *   1. f5_quant_w4_scales: every group's scale s into d_best_s [N][K/128]
 *      (double) and the bit pattern of max(s) into *d_smax_bits.  nalpha > 0:
 *      the MSE grid search of quant_linear_mse (ref/layer_fixed.py:981-1030)
 *      over the caller's alpha[] (numpy linspace(amin, 1, nalpha)),
 *      d_salience (nullable) = its per-channel error weights [K]
 *      (_salience_weights, ref/layer_fixed.py:943-978); nalpha = 0: the
 *      max|W|/7 rule of quantize_weights (ref/w4a8_ref.py:154-180).
 *   2. the caller sets e = ceil(log2(max s)) + 1 (ref/w4a8_ref.py:171; host
 *      libm, like the reference);
 *   3. f5_quant_w4_pack: m, eff and the codes; d_img [N][row stride]
 *      receives pack_ddr_rows' bytes (ref/w4a8_ref.py:349-370); d_w4 [N][K]
 *      and d_m [N][K/128] (both nullable) the unpacked w4 / m arrays.
 * sh is the fixed rule of final_shift (ref/w4a8_ref.py:177-179). */
int f5_quant_w4_scales(const void *d_w, int w_f64, int N, int K, int g, const double *alpha,
                       int nalpha, const double *d_salience, double *d_best_s,
                       uint64_t *d_smax_bits, void *stream);
int f5_quant_w4_pack(const void *d_w, int w_f64, int N, int K, int g, const double *d_best_s,
                     int e_shared, uint8_t *d_img, int8_t *d_w4, uint16_t *d_m,
                     void *stream);

/* Batched ref/w4a8_ref.py:254-289 matvec_y32 on the tensor cores (tcgen05
 * int8 MMA, int32 TMEM accumulators): y32[b][row] for B quantized inputs
 * d_x8 [B][K] against one packed image (d_w, 256-byte aligned), the way B
 * independent decode sequences share a weight matrix.  g = 128, K a multiple
 * of 1024 (<= 12288), 1 <= B <= 64.  d_ws: 256-byte aligned device workspace
 * of f5_batch_matvec_ws_bytes(N, K, B) bytes (0: unsupported shape).  d_p
 * (nullable): int64 p[b][row]; d_err: uint32 error word (bit 0 |y32| >= 2^31,
 * bit 1 a bounded device wait expired).  No counterpart in the reference,
 * which runs one sequence at a time: the batched form of matvec_y32. */
size_t f5_batch_matvec_ws_bytes(int N, int K, int B);
/* Pipeline trace of the batched GEMM (profiling aid): enable = 1 attaches a
 * zeroed device buffer of 10240 globaltimer words to every following batched
 * GEMM launch of the process (CTA 0 records, per stage, when it was issued
 * and unpacked, and per group when it was unpacked, multiplied, read back
 * and folded); enable = 0 copies up to cap words into out (nullable) and
 * detaches.  Synchronous. */
int f5_batch_trace(int enable, uint64_t *out, size_t cap);
int f5_batch_matvec_y32_dev(const uint8_t *d_w, int N, int K, int g, int sh, const int8_t *d_x8, int B,
                            int32_t *d_y32, int64_t *d_p, void *d_ws, size_t ws_bytes, uint32_t *d_err,
                            void *stream);

/* ---------------------------------------------------------------------------
 * Host-buffer entry points (allocate device scratch per call)
 * ------------------------------------------------------------------------- */

/* ref/w4a8_ref.py:254-289 matvec_y32 on a packed image (host pointers):
 * y32[N] and, if p != NULL, the int64 p[N]. */
int f5_matvec_y32_host(const uint8_t *img, int N, int K, int g, int sh,
                       const int8_t *x8, int32_t *y32, int64_t *p);

/* Allocation-free form of f5_matvec_y32_host, for callers that cannot call
 * cudaMalloc (a host whose device memory belongs to another allocator's
 * pool or arena, a loop that cannot take cudaMalloc/cudaFree's device
 * synchronisation).  No counterpart in the
 * reference: it is an extra deployment form of the matvec_y32 drop-in.
 * Stages everything in one fixed device array of F5_NOALLOC_SCRATCH_BYTES
 * that every GPU loading the library holds until exit; larger requests fail
 * with F5_EINVAL.  The first call on a device resolves the array's address
 * (make it before any stream capture).  Calls share the array: calls that
 * overlap on the GPU race.  Synchronous, legacy default stream. */
#define F5_NOALLOC_SCRATCH_BYTES (16u << 20)
int f5_matvec_y32_host_noalloc(const uint8_t *img, int N, int K, int g, int sh,
                               const int8_t *x8, int32_t *y32, int64_t *p);

/* ---------------------------------------------------------------------------
 * Model context: one GPU's resident integer Qwen3.5-9B model + decode state
 * ------------------------------------------------------------------------- */

typedef struct f5_ctx f5_ctx;

typedef struct f5_config {
  int abi_version;          /* F5_ABI_VERSION                                       */
  int n_layers;             /* 32 at 9B                                              */
  int vocab;                /* 248320 at 9B                                          */
  int max_T;                /* KV-cache capacity per attention layer (tokens)       */
  int norm_mode;            /* DeltaNet gated norm: 0 float64 host scale (layer_fixed
                               default, ref/layer_fixed.py:509-546), 1 integer EPS-NORM
                               (SEQ_NORM / seq_model epsnorm, :694-781)            */
  int world_size, rank;     /* row sharding (ref/seq_format.py:1177-1189); 1, 0     */
  const char *layer_types;  /* n_layers chars: 'D' linear_attention, 'A' full_attention
                               (copied at create)                                   */
} f5_config;

/* matrix slots (f5_ctx_upload_matrix): DeltaNet 0 in_qkv, 1 in_z, 2 in_b,
 * 3 in_a, 4 out; attention 0 q_proj, 1 k_proj, 2 v_proj, 3 o_proj; MLP
 * 8 gate, 9 up, 10 down; LM head: layer -1, slot 0 (ref/layer_fixed.py:
 * 1360-1375, 1455-1490, 1586-1595) */
enum f5_slot { F5_S_IN_QKV = 0, F5_S_IN_Z = 1, F5_S_IN_B = 2, F5_S_IN_A = 3, F5_S_OUT = 4,
               F5_S_Q = 0, F5_S_K = 1, F5_S_V = 2, F5_S_O = 3,
               F5_S_GATE = 8, F5_S_UP = 9, F5_S_DOWN = 10, F5_S_HEAD = 0 };

/* integer vector parameters (f5_ctx_upload_vector), as the reference's
 * quantized dicts hold them (ref/layer_fixed.py:1607-1651) */
enum f5_vec { F5_VEC_LN1 = 0, F5_VEC_LN2 = 1, F5_VEC_Q_NORM = 2, F5_VEC_K_NORM = 3,
              F5_VEC_CONV_W = 4 /* [CONV_DIM][4] */, F5_VEC_DT_BIAS = 5, F5_VEC_A = 6,
              F5_VEC_NORM_W = 7, F5_VEC_LN_F = 8 /* layer -1, (1+w) at Q3.12 */ };

/* device buffers readable with f5_ctx_read (debug taps and state) */
enum f5_buf { F5_BUF_X16 = 0, F5_BUF_QKV16 = 1, F5_BUF_Z16 = 2, F5_BUF_B16 = 3, F5_BUF_A16 = 4,
              F5_BUF_ON16 = 5, F5_BUF_QG16 = 6, F5_BUF_K16 = 7, F5_BUF_V16 = 8,
              F5_BUF_PROD64 = 9, F5_BUF_PROD16 = 10,
              F5_BUF_STATS = 11 /* uint64 [4], cumulative since f5_ctx_reset: [0] DeltaNet state
                                   writes clipped to int16 (the reference's state["sat"],
                                   ref/layer_fixed.py:1551,1569), [1] max |x| of every layer
                                   output, [2] layer-output words at the int16 rails (FxRunner
                                   resid_max / resid_clip, ref/fidelity_check.py:430-431), [3] 0 */,
              F5_BUF_DN_S = 12 /* int16 [32 heads][4][128 dk][32]: dv = 32 * quarter + i */, F5_BUF_DN_CONV = 13 /* int16 [8192][4] ring */,
              F5_BUF_DN_KH = 14, F5_BUF_K8 = 15, F5_BUF_KE = 16, F5_BUF_V8 = 17, F5_BUF_VE = 18,
              F5_BUF_KA = 19, F5_BUF_LOGITS = 20 /* int32 [vocab], see f5_ctx_set_logits */,
              F5_BUF_QKVC16 = 21 /* post-conv q|k|v of the last DeltaNet layer (graph engine) */,
              F5_BUF_GATES = 22 /* int32 [2][32] beta | decay of the last DeltaNet layer (graph engine) */ };

/* create / destroy (state zeroed, T = 0) */
int f5_ctx_create(const f5_config *cfg, int device, f5_ctx **out);
int f5_ctx_destroy(f5_ctx *ctx);

/* weights: a full pack_ddr_rows image of an N x K matrix (host; this rank's
 * row share is copied), or the seeded synthetic generator on the device.
 * Replaces the quantized dict {"w4","m","e","sh","g"} of ref/layer_fixed.py:
 * 1111 and the DDR images of ref/seq_model.py:305-452 (DDRWeights). */
int f5_ctx_upload_matrix(f5_ctx *ctx, int layer, int slot, const uint8_t *img, int N, int K, int g,
                         int e, int sh);
int f5_ctx_synth_matrix(f5_ctx *ctx, int layer, int slot, int N, int K, int g, int e, int sh,
                        uint64_t key_w, uint64_t key_m, int symmetric);
int f5_ctx_upload_vector(f5_ctx *ctx, int layer, int kind, const int64_t *v, int n);
/* int16 embedding table at Q.RS_F [vocab][4096] (ref/gen_model_script.py:546-552) */
int f5_ctx_upload_embedding(f5_ctx *ctx, const int16_t *emb, int vocab, int h);
int f5_ctx_synth_embedding(f5_ctx *ctx, uint64_t key_e);
/* RoPE tables [npos][128] = rope_tables_q15(pos) cos | sin (ref/layer_fixed.py:1333-1337) */
int f5_ctx_upload_rope(f5_ctx *ctx, const int16_t *tab, int npos);

/* state: zero every cache (ref/layer_fixed.py:1654-1666 new_cache_fx), T = 0 */
int f5_ctx_reset(f5_ctx *ctx);
int f5_ctx_set_position(f5_ctx *ctx, int T, int pos);
int f5_ctx_get_position(f5_ctx *ctx, int *T, int *pos);
/* also store the LM head's y32 logits (F5_BUF_LOGITS) each step: the
 * return value of ref/fidelity_check.py:423-448 FxRunner.step */
int f5_ctx_set_logits(f5_ctx *ctx, int on);
/* the context's CUDA stream (cudaStream_t) every launch of the context uses */
int f5_ctx_stream(f5_ctx *ctx, void **stream);
/* record the decode-step CUDA graph now (otherwise at the first step) */
int f5_ctx_prepare(f5_ctx *ctx);

/* TOPK-32 capture: the LM head's top-k unit (tb/scripts/gen_topk_cases.py:
 * 20-45, numpy model `Ref.push` :75-102) whose list the sampler of
 * sw/chat_seq.py:1776-1928 (`Sampler.pick(values, indices, e_x)`) consumes.
 * Elements arrive in array order with index = position.  No reference C
 * interface: the unit is RTL, read back through CSRs. */
typedef struct f5_topk32 {
  int32_t val[32];    /* value descending, ties by ascending index */
  int32_t idx[32];    /* index of each entry; -1 past count */
  int32_t count;      /* min(n, 32) */
  int32_t ovf_lit;    /* sticky: a rejected element tied entry[31] */
  int32_t ovf_disp;   /* sticky: ovf_lit, or a displaced element tied the new entry[31] */
  int32_t amax_idx;   /* the AMAX32 winner (first max) = entry 0; 0 when n = 0 */
  int32_t amax_val;
  int32_t e_x;        /* f5_ctx_topk: DYNQ8 exponent of the head's input, else 0 */
  int32_t n;          /* elements scanned */
} f5_topk32;
/* device scratch for f5_topk32_dev over n elements */
size_t f5_topk32_ws_bytes(long long n);
/* device pointers; out is device memory; runs on `stream` (cudaStream_t, NULL = default) */
int f5_topk32_dev(const int32_t *vals, long long n, void *ws, f5_topk32 *out, void *stream);
/* host pointers (allocates, copies, synchronises) */
int f5_topk32_host(const int32_t *vals, long long n, f5_topk32 *out);
/* the last step's TOPK-32 over the LM head's logits (needs
 * f5_ctx_set_logits(ctx, 1) before the step) and the head input's DYNQ8
 * exponent e_x (the sampler's dequant, sw/chat_seq.py:1842-1845), computed
 * from the final residual; single-GPU contexts */
int f5_ctx_topk(f5_ctx *ctx, f5_topk32 *out);

/* Decode engines (no reference counterpart: the reference has one sequencer).
 * F5_ENGINE_PERSISTENT runs each step as ONE cooperative launch of the
 * persistent decode kernel (one CTA per SM, weights streamed continuously
 * across op boundaries); F5_ENGINE_GRAPH replays the per-op kernel chain as a
 * CUDA graph.  Both compute the same integer law bit-exactly.  Default: the
 * persistent engine when the device can hold it resident, else the graph. */
enum f5_engine { F5_ENGINE_GRAPH = 0, F5_ENGINE_PERSISTENT = 1 };
int f5_ctx_set_engine(f5_ctx *ctx, int engine);
/* the engine the next step uses (builds its program if needed) */
int f5_ctx_get_engine(f5_ctx *ctx, int *engine);

/* Row-sharded decode across world_size GPUs (one process and context per
 * GPU; replaces the reference's 4-DIMM channel split, ref/seq_format.py:
 * 1177-1189 split_rows).  Each rank streams only its rows of every matrix
 * and its GEMV epilogues store their output words into every rank's buffers
 * (peer stores over NVLink, fused into the epilogue); the vector work is
 * replicated.  Before the first step, each rank exports its handle
 * (cudaIpcMemHandle_t, 64 bytes), the caller all-gathers them, and every
 * rank attaches all of them in rank order.  Persistent engine only. */
int f5_ctx_ipc_handle(f5_ctx *ctx, void *handle, size_t cap);
int f5_ctx_attach_peers(f5_ctx *ctx, const void *handles, int n);

/* Timeline of one persistent step (no reference counterpart: profiling aid).
 * Runs one greedy step (caches advance) with every CTA recording the device
 * globaltimer (ns) at 8 marks of each op: out[(cta * nops + op) * 8 + k],
 * k = 0 start (after the grid barrier), 1 end, 2..6 op phases, 7 arrival at
 * the next grid barrier (0 where a CTA has no such phase).  With out == NULL
 * only *grid and *nops are returned; otherwise cap >= grid * nops * 8.
 * The step runs on a separately compiled instance of the persistent kernel
 * that carries the marks (the step kernel itself has none): same program and
 * results, a few percent slower. */
int f5_ctx_trace_step(f5_ctx *ctx, uint64_t *out, size_t cap, int *grid, int *nops);

/* One full model step from a host token id: embedding row, every layer,
 * final RMSNorm, DYNQ8, LM head, argmax (first max wins).  Replaces
 * ref/fidelity_check.py:423-448 FxRunner.step and the token loop of
 * ref/gen_model_script.py:602-650.  Caches advance by one token (T += 1). */
int f5_decode_step(f5_ctx *ctx, int32_t tok, int32_t pos, int32_t *next_tok, int32_t *max_logit);
/* n greedy steps on the device without host round trips: each step feeds
 * its argmax to the next (pos and T advance); read the last with f5_ctx_sync */
int f5_decode_launch(f5_ctx *ctx, int n_steps, void *stream_unused);
/* Prefill: n steps whose input tokens are tokens[0..n) (host array), from
 * the context's current position, without a host round trip between steps
 * (the reference prefills a prompt the same way, one token per step:
 * sw/chat_client.py:21, ref/fidelity_check.py:423-448 per token).  After
 * it, the next device-fed step (f5_decode_launch) starts from the argmax of
 * the last prompt step; f5_ctx_sync returns it.  Asynchronous. */
int f5_decode_prefill(f5_ctx *ctx, const int32_t *tokens, int n);
int f5_ctx_sync(f5_ctx *ctx, int32_t *last_tok, int32_t *max_logit);

/* Run `reps` decode steps eagerly with a CUDA event pair around every kernel
 * launch (measurement only; caches advance).  out[8] per step (averaged):
 * {GEMV ms, GEMV algorithmic weight bytes, GEMV launches, DeltaNet-step ms,
 *  attention ms, other ms, sum of launch ms, launches}. */
int f5_ctx_time_step(f5_ctx *ctx, int reps, double *out, int nout);

/* One decoder layer on a host residual vector at cache length T and RoPE
 * position pos (ref/layer_fixed.py:1669-1677 layer_decode_fx); the layer's
 * cache is updated in place (KV slot T / conv window / state). */
int f5_layer_step(f5_ctx *ctx, int layer, int16_t *x16_inout, int T, int pos);

/* State I/O in the reference's cache layout (ref/layer_fixed.py:1654-1666
 * new_cache_fx, the caches layer_decode_fx mutates, :1400-1401 and
 * :1522-1569), one layer at a time:
 *   DeltaNet layer: S int16 [32][128][128] (head, dk, dv), then the conv
 *     window int64 [8192][3], oldest first (cache["S"], cache["conv"]);
 *   attention layer at T tokens: k8 int8 [T][4][256], ke int8 [T][4],
 *     v8 int8 [T][4][256], ve int8 [T][4] (cache["k"][t][h] = (k8, ke),
 *     cache["v"][t][h] = (v8, ve)).
 * f5_state_bytes: image size (0 for a bad layer); f5_state_save: the layer's
 * image at the context's current T; f5_state_load: write the layer's state
 * from an image of T tokens (then set T / pos with f5_ctx_set_position). */
size_t f5_state_bytes(f5_ctx *ctx, int layer, int T);
int f5_state_save(f5_ctx *ctx, int layer, void *dst, size_t bytes);
int f5_state_load(f5_ctx *ctx, int layer, const void *src, size_t bytes, int T);

/* raw device buffer copies (enum f5_buf); bytes must equal the buffer size */
int f5_ctx_read(f5_ctx *ctx, int what, int layer, void *dst, size_t bytes);
int f5_ctx_write(f5_ctx *ctx, int what, int layer, const void *src, size_t bytes);

/* ---------------------------------------------------------------------------
 * Batched decode: B independent greedy sequences over one loaded model
 * ------------------------------------------------------------------------- */

/* The reference decodes one sequence at a time (ref/fidelity_check.py:
 * 404-448); a batched context runs B such independent decode steps at once.
 * It borrows the weights of a fully loaded model context `model` (which must
 * outlive it, world_size 1, g = 128 images) and owns B sequences' decode
 * state (DeltaNet states and conv windows, KV caches of max_T tokens, T and
 * pos), all zero at creation.  Every projection runs as a W4A8 GEMM of the B
 * quantized inputs on the tensor cores; per sequence, every result equals
 * the single-sequence step's bit for bit.  1 <= batch <= 64. */
typedef struct f5_bctx f5_bctx;
int f5_bctx_create(f5_ctx *model, int batch, int max_T, f5_bctx **out);
int f5_bctx_destroy(f5_bctx *bctx);
int f5_bctx_reset(f5_bctx *bctx);                                /* all states zero, T = pos = 0 */
int f5_bctx_set_position(f5_bctx *bctx, int seq, int T, int pos); /* seq = -1: every sequence */
int f5_bctx_get_position(f5_bctx *bctx, int seq, int *T, int *pos);
/* one step of every sequence: tok[B] in, next_tok[B] / max_logit[B] out
 * (nullable); advances each sequence's T and pos by one */
int f5_bctx_step(f5_bctx *bctx, const int32_t *tok, int32_t *next_tok, int32_t *max_logit);
/* Layer-major prompt ingestion into sequence seq: the n prompt tokens go
 * through the model in chunks of up to `batch` tokens, each chunk's tokens
 * being the columns of every projection GEMM (one read of every weight
 * image per chunk instead of one per token), while the conv windows, the
 * DeltaNet recurrences and the KV appends run token by token in order.  The
 * sequence's state, T and pos end exactly as n decode steps leave them
 * (sw/chat_client.py:21 feeds a prompt one step at a time); next_tok /
 * max_logit (nullable) receive the argmax after the last prompt token, and
 * the sequence's next step input is set to it.  Other sequences are not
 * touched. */
int f5_bctx_prefill(f5_bctx *bctx, int seq, const int32_t *tokens, int n, int32_t *next_tok,
                    int32_t *max_logit);
/* enqueue n greedy steps (each sequence fed its own argmax), no host sync */
int f5_bctx_launch(f5_bctx *bctx, int n_steps);
int f5_bctx_sync(f5_bctx *bctx, int32_t *last_tok, int32_t *max_logit);
int f5_bctx_stream(f5_bctx *bctx, void **stream);
/* device time of one eager batched step per kernel class, averaged over reps
 * steps (CUDA events around every launch; each step advances every
 * sequence): out[0..5] ms of prologue / GEMM / epilogue / DeltaNet /
 * attention / other kernels, out[6..11] their algorithmic weight bytes,
 * out[12] launches per step, out[13] the sum of the kernel times (nout >= 14) */
int f5_bctx_time_step(f5_bctx *bctx, int reps, double *out, int nout);
/* sequence seq's copy of an f5_buf buffer (same sizes as f5_ctx_read): the
 * state buffers of a layer, and the activations of the last layer that wrote
 * them (X16, QKV16, Z16, B16, A16, ON16, QG16, K16, V16, PROD64, PROD16) */
/* also store the LM head's y32 logits of every sequence each step
 * (F5_BUF_LOGITS, per sequence), as f5_ctx_set_logits does for one */
int f5_bctx_set_logits(f5_bctx *bctx, int on);
/* the last step's TOPK-32 capture of every sequence (out: batch entries)
 * with each sequence's head-input exponent e_x: the candidate sets that
 * sw/chat_seq.py:1776-1928 Sampler.pick draws from, per sequence */
int f5_bctx_topk(f5_bctx *bctx, f5_topk32 *out);
int f5_bctx_read(f5_bctx *bctx, int seq, int what, int layer, void *dst, size_t bytes);
int f5_bctx_write(f5_bctx *bctx, int seq, int what, int layer, const void *src, size_t bytes);

#ifdef __cplusplus
}
#endif
#endif /* F5B200_H */
