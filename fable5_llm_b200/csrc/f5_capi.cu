// C ABI: stateless entry points (device-pointer kernels, host-buffer matvec).
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "../../include/f5b200.h"
#include "f5_capi_util.h"
#include "f5_kernels.cuh"
#include "f5_topk.cuh"

namespace f5 {
cudaError_t launch_synth_w4(uint8_t *, long long, int, int, long long, uint64_t, uint64_t, int,
                            cudaStream_t);
cudaError_t launch_synth_emb(int16_t *, long long, int, long long, uint64_t, cudaStream_t);

static thread_local char g_err[512] = "";

int set_error(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_status(cudaError_t e, const char *where) {
  if (e == cudaSuccess) return F5_OK;
  (void)cudaGetLastError();
  return set_error(e == cudaErrorMemoryAllocation ? F5_ENOMEM : F5_ECUDA, "%s: %s", where,
                   cudaGetErrorString(e));
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int check_matrix_shape(int N, int K, int g) {
  if (N <= 0 || K <= 0 || (K % 128) != 0 || K > 12288)
    return set_error(F5_EINVAL, "matrix shape N=%d K=%d: K must be a multiple of 128 in [128, 12288]", N, K);
  if (g != 128 && g != 64) return set_error(F5_EINVAL, "group size g=%d has no wire format (128 or 64)", g);
  return F5_OK;
}

int row_stride(int K, int g) { return (K / 128 + (K / g + 31) / 32) * 64; }

}  // namespace f5

using namespace f5;

extern "C" {

int f5_abi_version(void) { return F5_ABI_VERSION; }

const char *f5_status_string(int s) {
  switch (s) {
    case F5_OK: return "ok";
    case F5_EINVAL: return "invalid argument";
    case F5_ECUDA: return "CUDA error";
    case F5_ENOMEM: return "out of device memory";
    case F5_ETIMEOUT: return "device wait timed out";
    case F5_EOVERFLOW: return "range assertion failed";
    case F5_ESTATE: return "invalid state";
    case F5_ENCCL: return "collective failed";
    default: return "unknown status";
  }
}

int f5_last_error(char *buf, size_t len) {
  if (!buf || !len) return F5_EINVAL;
  strncpy(buf, g_err, len - 1);
  buf[len - 1] = 0;
  return F5_OK;
}

int f5_gemv_dev(const f5_gemv_seg *segs, int nseg, int K, int g, int sh, const int8_t *d_x8,
                const int *d_xmeta, unsigned long long *d_argmax, uint32_t *d_err, int max_blocks,
                int pdl, void *stream) {
  if (!segs || nseg < 1 || nseg > GEMV_MAX_SEG || !d_x8 || !d_err)
    return set_error(F5_EINVAL, "f5_gemv_dev: bad segment list / null x8 or err");
  GemvArgs a = {};
  a.nseg = nseg;
  a.K = K;
  a.g = g;
  a.sh = sh;
  a.stride = row_stride(K, g);
  a.x8 = d_x8;
  a.xmeta = d_xmeta;
  a.argmax_key = d_argmax;
  a.err = d_err;
  int units = 0;
  for (int i = 0; i < nseg; ++i) {
    const f5_gemv_seg &s = segs[i];
    int st = check_matrix_shape(s.rows, K, g);
    if (st) return st;
    if (!s.w || (!s.out && s.mode != F5_GM_ARGMAX)) return set_error(F5_EINVAL, "f5_gemv_dev: null segment pointer");
    if ((reinterpret_cast<uintptr_t>(s.w) & 15) || (reinterpret_cast<uintptr_t>(s.w2) & 15))
      return set_error(F5_EINVAL, "f5_gemv_dev: weight images must be 16-byte aligned (bulk copies)");
    if (s.mode < 0 || s.mode > F5_GM_ARGMAX) return set_error(F5_EINVAL, "f5_gemv_dev: bad mode %d", s.mode);
    if (s.mode == F5_GM_SILU_MUL && !s.w2) return set_error(F5_EINVAL, "f5_gemv_dev: SILU_MUL needs w2");
    if (s.mode == F5_GM_ARGMAX && !d_argmax) return set_error(F5_EINVAL, "f5_gemv_dev: ARGMAX needs d_argmax");
    GemvSeg &d = a.seg[i];
    d.w = s.w;
    d.w2 = s.w2;
    d.out = s.out;
    d.p_out = s.p_out;
    d.rows = s.rows;
    d.unit_begin = units;
    d.e = s.e;
    d.e2 = s.e2;
    d.out_f = s.out_f;
    d.out_f2 = s.out_f2;
    d.mode = s.mode;
    d.out_row0 = s.out_row0;
    units += s.rows;   // a unit is one row (SILU_MUL: one gate/up row pair)
  }
  a.total_units = units;
  if (max_blocks <= 0) max_blocks = sm_count();
  return cuda_status(launch_gemv(a, (cudaStream_t)stream, pdl != 0, max_blocks), "f5_gemv_dev");
}

int f5_rmsnorm_dynq8_dev(const int16_t *d_x16, const int32_t *d_w, int n, int in_f, int one_plus,
                         int16_t *d_xn, int8_t *d_x8, int *d_meta, void *stream) {
  if (!d_x16 || !d_w || !d_x8 || !d_meta) return set_error(F5_EINVAL, "f5_rmsnorm_dynq8_dev: null pointer");
  if (n <= 0 || n > 4096 || (n & (n - 1)))
    return set_error(F5_EINVAL, "rmsnorm: N=%d is not a power of two <= 4096 (ref/layer_fixed.py:653-678)", n);
  NormArgs a = {};
  a.x16 = d_x16;
  a.w = d_w;
  a.n = n;
  a.in_f = in_f;
  a.one_plus = one_plus;
  a.xn_out = d_xn;
  a.out.x8 = d_x8;
  a.out.meta = d_meta;
  return cuda_status(launch_rmsnorm_dynq8(a, (cudaStream_t)stream, false), "f5_rmsnorm_dynq8_dev");
}

int f5_dynq8_dev(const int16_t *d_x16, int n, int in_f, int8_t *d_x8, int *d_meta, void *stream) {
  if (!d_x16 || !d_x8 || !d_meta) return set_error(F5_EINVAL, "f5_dynq8_dev: null pointer");
  if (n <= 0 || n > 12288) return set_error(F5_EINVAL, "f5_dynq8_dev: n=%d outside [1, 12288]", n);
  Dynq8Args a = {};
  a.x16 = d_x16;
  a.n = n;
  a.in_f = in_f;
  a.out.x8 = d_x8;
  a.out.meta = d_meta;
  return cuda_status(launch_dynq8(a, (cudaStream_t)stream, false), "f5_dynq8_dev");
}

int f5_prim_dev(int op, const int64_t *d_in, const int64_t *d_in2, int64_t *d_out, int64_t *d_out2,
                int n, int arg0, int arg1, void *stream) {
  if (!d_in || !d_out || n < 0) return set_error(F5_EINVAL, "f5_prim_dev: bad arguments");
  if (op < 0 || op > F5_PR_EXP2_FRAC) return set_error(F5_EINVAL, "f5_prim_dev: bad op %d", op);
  if ((op == F5_PR_DN_NORM_SCALE || op == F5_PR_EPS_NORM_SCALE) && !d_in2)
    return set_error(F5_EINVAL, "f5_prim_dev: norm scale needs per-element k");
  return cuda_status(launch_prim(op, d_in, d_in2, d_out, d_out2, n, arg0, arg1, (cudaStream_t)stream),
                     "f5_prim_dev");
}

int f5_synth_w4_dev(uint8_t *d_img, long long nrows, int K, int g, long long row0, uint64_t key_w,
                    uint64_t key_m, int symmetric, void *stream) {
  if (!d_img) return set_error(F5_EINVAL, "f5_synth_w4_dev: null image");
  int st = check_matrix_shape(nrows > 0 ? 1 : 0, K, g);
  if (st) return st;
  return cuda_status(launch_synth_w4(d_img, nrows, K, g, row0, key_w, key_m, symmetric, (cudaStream_t)stream),
                     "f5_synth_w4_dev");
}

int f5_synth_emb_dev(int16_t *d_emb, long long nrows, int H, long long row0, uint64_t key_e, void *stream) {
  if (!d_emb || H <= 0 || (H % 4)) return set_error(F5_EINVAL, "f5_synth_emb_dev: bad arguments");
  return cuda_status(launch_synth_emb(d_emb, nrows, H, row0, key_e, (cudaStream_t)stream), "f5_synth_emb_dev");
}

int f5_matvec_y32_host(const uint8_t *img, int N, int K, int g, int sh, const int8_t *x8, int32_t *y32,
                       int64_t *p) {
  if (!img || !x8 || !y32) return set_error(F5_EINVAL, "f5_matvec_y32_host: null pointer");
  int st = check_matrix_shape(N, K, g);
  if (st) return st;
  const size_t stride = (size_t)row_stride(K, g);
  uint8_t *d_img = nullptr;
  int8_t *d_x8 = nullptr;
  int32_t *d_y = nullptr;
  int64_t *d_p = nullptr;
  uint32_t *d_err = nullptr;
  uint32_t herr = 0;
  cudaError_t e = cudaSuccess;
  f5_gemv_seg s = {};
  int rc = F5_OK;
#define F5_TRY(x)                          \
  do {                                     \
    e = (x);                               \
    if (e != cudaSuccess) goto done;       \
  } while (0)
  F5_TRY(cudaMalloc(&d_img, stride * N));
  F5_TRY(cudaMalloc(&d_x8, K));
  F5_TRY(cudaMalloc(&d_y, sizeof(int32_t) * N));
  if (p) F5_TRY(cudaMalloc(&d_p, sizeof(int64_t) * N));
  F5_TRY(cudaMalloc(&d_err, sizeof(uint32_t)));
  F5_TRY(cudaMemcpy(d_img, img, stride * N, cudaMemcpyHostToDevice));
  F5_TRY(cudaMemcpy(d_x8, x8, K, cudaMemcpyHostToDevice));
  F5_TRY(cudaMemset(d_err, 0, sizeof(uint32_t)));
  s.w = d_img;
  s.out = d_y;
  s.p_out = d_p;
  s.rows = N;
  s.mode = F5_GM_Y32;
  rc = f5_gemv_dev(&s, 1, K, g, sh, d_x8, nullptr, nullptr, d_err, 0, 0, nullptr);
  if (rc) goto done;
  F5_TRY(cudaMemcpy(y32, d_y, sizeof(int32_t) * N, cudaMemcpyDeviceToHost));
  if (p) F5_TRY(cudaMemcpy(p, d_p, sizeof(int64_t) * N, cudaMemcpyDeviceToHost));
  F5_TRY(cudaMemcpy(&herr, d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  if (herr & DERR_Y32_OVERFLOW) rc = set_error(F5_EOVERFLOW, "y32 overflow -- sh miscomputed (ref/w4a8_ref.py:288)");
  else if (herr & DERR_TIMEOUT) rc = set_error(F5_ETIMEOUT, "a bounded device wait gave up");
done:
#undef F5_TRY
  if (e != cudaSuccess) rc = cuda_status(e, "f5_matvec_y32_host");
  cudaFree(d_img);
  cudaFree(d_x8);
  cudaFree(d_y);
  cudaFree(d_p);
  cudaFree(d_err);
  return rc;
}


// ---------------------------------------------------------------------------
// TOPK-32 capture
// ---------------------------------------------------------------------------
size_t f5_topk32_ws_bytes(long long n) { return f5::topk32_ws_bytes(n); }

int f5_topk32_dev(const int32_t *vals, long long n, void *ws, f5_topk32 *out, void *stream) {
  if (n < 0 || n > 0x7FFFFFFFll) return set_error(F5_EINVAL, "f5_topk32_dev: n=%lld outside [0, 2^31)", n);
  if ((n > 0 && !vals) || !ws || !out) return set_error(F5_EINVAL, "f5_topk32_dev: null pointer");
  return cuda_status(f5::launch_topk32(vals, n, ws, out, nullptr, (cudaStream_t)stream), "f5_topk32_dev");
}

int f5_topk32_host(const int32_t *vals, long long n, f5_topk32 *out) {
  if (n < 0 || n > 0x7FFFFFFFll) return set_error(F5_EINVAL, "f5_topk32_host: n=%lld outside [0, 2^31)", n);
  if ((n > 0 && !vals) || !out) return set_error(F5_EINVAL, "f5_topk32_host: null pointer");
  int32_t *d_v = nullptr;
  void *d_ws = nullptr;
  f5_topk32 *d_out = nullptr;
  cudaError_t e = cudaSuccess;
#define F5_TRY(x)                          \
  do {                                     \
    e = (x);                               \
    if (e != cudaSuccess) goto done;       \
  } while (0)
  F5_TRY(cudaMalloc(&d_v, sizeof(int32_t) * (size_t)(n > 0 ? n : 1)));
  F5_TRY(cudaMalloc(&d_ws, f5::topk32_ws_bytes(n)));
  F5_TRY(cudaMalloc(&d_out, sizeof(f5_topk32)));
  if (n > 0) F5_TRY(cudaMemcpy(d_v, vals, sizeof(int32_t) * (size_t)n, cudaMemcpyHostToDevice));
  F5_TRY(f5::launch_topk32(d_v, n, d_ws, d_out, nullptr, 0));
  F5_TRY(cudaMemcpy(out, d_out, sizeof(f5_topk32), cudaMemcpyDeviceToHost));
done:
#undef F5_TRY
  cudaFree(d_v);
  cudaFree(d_ws);
  cudaFree(d_out);
  return e == cudaSuccess ? F5_OK : cuda_status(e, "f5_topk32_host");
}
}  // extern "C"

// ---------------------------------------------------------------------------
// batched matvec_y32 on the tensor cores
// ---------------------------------------------------------------------------
#include "f5_batch.cuh"

namespace {
struct BmLayout {
  int NG, Bp, S, tiles;
  size_t xt, xmeta, p, total;
};
size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }
bool bm_layout(int N, int K, int B, BmLayout &L) {
  if (N <= 0 || K <= 0 || K % 1024 || K > 12288 || B < 1 || B > 64) return false;
  L.NG = K / 128;
  L.Bp = B <= 16 ? 16 : (B <= 32 ? 32 : 64);
  L.tiles = (N + f5::BG_TILE - 1) / f5::BG_TILE;
  L.S = f5::bgemm_splits(L.tiles, L.NG, f5::sm_count(), false);
  size_t o = 0;
  L.xt = o; o += al256((size_t)L.NG * L.Bp * 128);
  L.xmeta = o; o += al256((size_t)L.Bp * 2 * 4);
  L.p = o; o += al256((size_t)L.S * L.Bp * N * 8);
  L.total = o;
  return true;
}
}  // namespace

extern "C" {

int f5_batch_trace(int enable, uint64_t *out, size_t cap) {
  unsigned long long *&tb = bgemm_trace_buffer();
  if (enable) {
    if (!tb) {
      cudaError_t e = cudaMalloc(&tb, BG_TRACE_WORDS * sizeof(unsigned long long));
      if (e != cudaSuccess) { tb = nullptr; return cuda_status(e, "f5_batch_trace"); }
    }
    return cuda_status(cudaMemset(tb, 0, BG_TRACE_WORDS * sizeof(unsigned long long)), "f5_batch_trace");
  }
  if (!tb) return set_error(F5_ESTATE, "f5_batch_trace: tracing is not enabled");
  int rc = F5_OK;
  if (out) {
    const size_t n = cap < (size_t)BG_TRACE_WORDS ? cap : (size_t)BG_TRACE_WORDS;
    rc = cuda_status(cudaMemcpy(out, tb, n * sizeof(uint64_t), cudaMemcpyDeviceToHost), "f5_batch_trace");
  }
  cudaFree(tb);
  tb = nullptr;
  return rc;
}

size_t f5_batch_matvec_ws_bytes(int N, int K, int B) {
  BmLayout L;
  return bm_layout(N, K, B, L) ? L.total : 0;
}

int f5_batch_matvec_y32_dev(const uint8_t *d_w, int N, int K, int g, int sh, const int8_t *d_x8, int B,
                            int32_t *d_y32, int64_t *d_p, void *d_ws, size_t ws_bytes, uint32_t *d_err,
                            void *stream) {
  int st = check_matrix_shape(N, K, g);
  if (st) return st;
  BmLayout L;
  if (g != 128 || !bm_layout(N, K, B, L))
    return set_error(F5_EINVAL, "f5_batch_matvec_y32_dev: needs g=128, K a multiple of 1024, 1 <= B <= 64");
  if (!d_w || !d_x8 || !d_y32 || !d_ws || !d_err) return set_error(F5_EINVAL, "f5_batch_matvec_y32_dev: null pointer");
  if (ws_bytes < L.total) return set_error(F5_EINVAL, "f5_batch_matvec_y32_dev: workspace %zu < %zu bytes", ws_bytes, L.total);
  if ((reinterpret_cast<uintptr_t>(d_w) | reinterpret_cast<uintptr_t>(d_ws)) & 255)
    return set_error(F5_EINVAL, "f5_batch_matvec_y32_dev: image and workspace must be 256-byte aligned");
  uint8_t *ws = static_cast<uint8_t *>(d_ws);
  cudaStream_t cs = (cudaStream_t)stream;
  // padded sequences read zero x tiles
  cudaError_t e = cudaMemsetAsync(ws + L.xt, 0, L.xmeta - L.xt, cs);   // padded sequences: zero x
  if (e != cudaSuccess) return cuda_status(e, "f5_batch_matvec_y32_dev");
  BprepArgs pa = {};
  pa.pro.mode = PRO_X8;
  pa.K = K; pa.NG = L.NG; pa.B = B; pa.Bp = L.Bp;
  pa.x8_in = d_x8;
  pa.xmeta = reinterpret_cast<int *>(ws + L.xmeta);
  pa.xt = reinterpret_cast<int8_t *>(ws + L.xt);
  pa.err = d_err;
  if ((e = launch_bprep(pa, cs, false)) != cudaSuccess) return cuda_status(e, "f5_batch_matvec_y32_dev/prep");
  BgemmArgs ga = {};
  ga.nseg = 1;
  ga.seg[0].w = d_w;
  ga.seg[0].rows = N;
  ga.ntiles = L.tiles;
  ga.K = K; ga.NG = L.NG; ga.stride = row_stride(K, g); ga.sh = sh;
  ga.S = L.S; ga.B = B; ga.Bp = L.Bp;
  ga.xt = pa.xt;
  ga.p = reinterpret_cast<int64_t *>(ws + L.p);
  ga.ptot = N;
  ga.err = d_err;
  if ((e = launch_bgemm(ga, cs, false, sm_count())) != cudaSuccess) return cuda_status(e, "f5_batch_matvec_y32_dev/gemm");
  BepiArgs ea = {};
  ea.g.nseg = 1;
  ea.g.K = K; ea.g.sh = sh; ea.g.err = d_err;
  ea.g.total_units = N;
  ea.g.seg[0].out = d_y32;
  ea.g.seg[0].p_out = d_p;
  ea.g.seg[0].rows = N;
  ea.g.seg[0].mode = GM_Y32;
  ea.bs[0].out_bs = (long long)N * 4;
  ea.bs[0].pout_bs = (long long)N * 8;
  ea.S = L.S; ea.B = B; ea.Bp = L.Bp; ea.ptot = N;
  ea.p = ga.p;
  ea.xmeta = pa.xmeta;
  if ((e = launch_bepi(ea, cs, false)) != cudaSuccess) return cuda_status(e, "f5_batch_matvec_y32_dev/epi");
  return F5_OK;
}

}  // extern "C"
