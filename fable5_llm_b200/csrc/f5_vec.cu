// Vector kernels: fused RMSNorm + DYNQ8, standalone DYNQ8, primitive eval.
#include "f5_block.cuh"
#include "f5_kernels.cuh"

namespace f5 {

constexpr int NORM_THREADS = 1024;
constexpr int NORM_MAXPT = 4;      // n <= 4096
constexpr int DQ_MAXPT = 12;       // n <= 12288

// ref/layer_fixed.py:1242-1278 rmsnorm_fx fused with ref/fixedpoint.py:24-33
// dyn_quant_i8 on its output.  One CTA (the vector is 8 KB).  When a token
// pointer is given the input is the embedding row emb[tok] (model step
// start, ref/fidelity_check.py:428), which is also copied to x16_store.
__global__ void __launch_bounds__(NORM_THREADS) k_rmsnorm_dynq8(const __grid_constant__ NormArgs a) {
  __shared__ long long red[32];
  __shared__ long long s_r;
  __shared__ int s_e;
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int n = a.n, tid = threadIdx.x;
  const int16_t *src = a.x16;
  if (a.emb) src = a.emb + (size_t)(*a.tok) * n;
  long long xv[NORM_MAXPT];
  long long ss = 0;
#pragma unroll
  for (int j = 0; j < NORM_MAXPT; ++j) {
    const int i = tid + j * NORM_THREADS;
    xv[j] = i < n ? (long long)src[i] : 0;
    ss += xv[j] * xv[j];
    if (a.emb && a.x16_store && i < n) a.x16_store[i] = (int16_t)xv[j];
  }
  ss = block_sum_ll(ss, red);
  if (tid == 0) {
    const int nbits = 31 - __clz(n);
    int64_t r; int e;
    rsqrt_q((uint64_t)(ss == 0 ? 1 : ss), 2 * a.in_f + nbits, r, e);
    s_r = r; s_e = e;
  }
  __syncthreads();
  const long long r = s_r;
  const int e = s_e;
  long long xn[NORM_MAXPT];
  unsigned long long mx = 0;
#pragma unroll
  for (int j = 0; j < NORM_MAXPT; ++j) {
    const int i = tid + j * NORM_THREADS;
    if (i < n) {
      long long y = rshr(xv[j] * r, 30 - e);
      y = clip(y, -(1ll << 32), (1ll << 32) - 1);
      const long long sc = (long long)a.w[i] + (a.one_plus ? (1 << 14) : 0);
      xn[j] = clip16(rshr(y * sc, 14));
      if (a.xn_out) a.xn_out[i] = (int16_t)xn[j];
      const unsigned long long m = uabs(xn[j]);
      mx = m > mx ? m : mx;
    } else {
      xn[j] = 0;
    }
  }
  mx = block_max_ull(mx, reinterpret_cast<unsigned long long *>(red));
  const int ex = dynq8_e(mx);
#pragma unroll
  for (int j = 0; j < NORM_MAXPT; ++j) {
    const int i = tid + j * NORM_THREADS;
    if (i < n) a.out.x8[i] = (int8_t)dynq8_apply(xn[j], ex);
  }
  if (tid == 0) { a.out.meta[0] = ex; a.out.meta[1] = a.in_f; }
}

// ref/fixedpoint.py:24-33 dyn_quant_i8 of an int16 vector (n <= 12288)
__global__ void __launch_bounds__(NORM_THREADS) k_dynq8(const __grid_constant__ Dynq8Args a) {
  __shared__ unsigned long long red[32];
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x;
  int32_t xv[DQ_MAXPT];
  unsigned long long mx = 0;
#pragma unroll
  for (int j = 0; j < DQ_MAXPT; ++j) {
    const int i = tid + j * NORM_THREADS;
    xv[j] = i < a.n ? (int32_t)a.x16[i] : 0;
    const unsigned long long m = uabs(xv[j]);
    mx = m > mx ? m : mx;
  }
  mx = block_max_ull(mx, red);
  const int ex = dynq8_e(mx);
#pragma unroll
  for (int j = 0; j < DQ_MAXPT; ++j) {
    const int i = tid + j * NORM_THREADS;
    if (i < a.n) a.out.x8[i] = (int8_t)dynq8_apply(xv[j], ex);
  }
  if (tid == 0) { a.out.meta[0] = ex; a.out.meta[1] = a.in_f; }
}

static cudaError_t launch1(const void *fn, void **args, int threads, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(threads);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_rmsnorm_dynq8(const NormArgs &a, cudaStream_t st, bool pdl) {
  if (a.n > NORM_THREADS * NORM_MAXPT || a.n <= 0 || (a.n & (a.n - 1))) return cudaErrorInvalidValue;
  NormArgs c = a;
  void *args[] = {&c};
  return launch1((const void *)k_rmsnorm_dynq8, args, NORM_THREADS, st, pdl);
}

cudaError_t launch_dynq8(const Dynq8Args &a, cudaStream_t st, bool pdl) {
  if (a.n > NORM_THREADS * DQ_MAXPT || a.n <= 0) return cudaErrorInvalidValue;
  Dynq8Args c = a;
  void *args[] = {&c};
  return launch1((const void *)k_dynq8, args, NORM_THREADS, st, pdl);
}

// ---- elementwise primitive evaluation (tests of the integer law) ----
__global__ void k_prim(int op, const int64_t *in, const int64_t *in2, int64_t *out,
                       int64_t *out2, int n, int arg0, int arg1) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int64_t x = in[i];
    int64_t r = 0, r2 = 0;
    switch (op) {
      case PR_RSHR: r = rshr(x, in2 ? (int)in2[i] : arg0); break;
      case PR_SIGMOID: r = sigmoid_q(x); break;
      case PR_SOFTPLUS: r = softplus_q(x); break;
      case PR_SILU: r = silu_q(x); break;
      case PR_EXP_NEG: r = exp_neg_q(x); break;
      case PR_EXP2_FRAC: r = exp2_frac_q16(x); break;
      case PR_RSQRT: { int64_t rr; int e; rsqrt_q((uint64_t)x, in2 ? (int)in2[i] : arg0, rr, e); r = rr; r2 = e; } break;
      case PR_RECIP: { int64_t rr; int e; recip_q((uint64_t)x, in2 ? (int)in2[i] : arg0, rr, e); r = rr; r2 = e; } break;
      case PR_BF_SHIFT: r = bf_shift(uabs(x)); break;
      case PR_DYNQ8_E: r = dynq8_e(uabs(x)); break;
      case PR_DN_NORM_SCALE: r = dn_norm_scale(x, (int)in2[i], arg0); break;
      case PR_EPS_NORM_SCALE: r = eps_norm_scale(x, (int)in2[i], arg0); break;
      default: break;
    }
    out[i] = r;
    if (out2) out2[i] = r2;
  }
}

cudaError_t launch_prim(int op, const int64_t *in, const int64_t *in2, int64_t *out,
                        int64_t *out2, int n, int arg0, int arg1, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  k_prim<<<blocks, 256, 0, st>>>(op, in, in2, out, out2, n, arg0, arg1);
  return cudaGetLastError();
}

}  // namespace f5
