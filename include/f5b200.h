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

/* ---------------------------------------------------------------------------
 * Host-buffer entry points (allocate device scratch per call)
 * ------------------------------------------------------------------------- */

/* ref/w4a8_ref.py:254-289 matvec_y32 on a packed image (host pointers):
 * y32[N] and, if p != NULL, the int64 p[N]. */
int f5_matvec_y32_host(const uint8_t *img, int N, int K, int g, int sh,
                       const int8_t *x8, int32_t *y32, int64_t *p);

#ifdef __cplusplus
}
#endif
#endif /* F5B200_H */
