// W4 group quantization of a float weight matrix on the GPU, written straight
// into the packed row format that the decode engines keep resident in HBM.
//
// Restates, bit for bit:
//  * quant_linear_mse (ref/layer_fixed.py:981-1030): per group of g = 128
//    weights, smax = max(max|w|, 1e-12); for each alpha of the grid
//    linspace(amin, 1, nalpha) the scale s = (smax / 7) * alpha, the codes
//    q = clip(rint(w / s), -8, 7) and the error sum((q s - w)^2) (optionally
//    weighted per input channel); the first alpha with the strictly smallest
//    error wins;
//  * quantize_weights (ref/w4a8_ref.py:154-180): the same with the single
//    scale smax / 7 (no search);
//  * the shared tail of both: m = clip(rint(s 2^(15-e)), 1, 65535),
//    eff = m 2^(e-15), w4 = clip(rint(w / eff), -8, 7), packed as
//    pack_ddr_rows (ref/w4a8_ref.py:331-370: low nibble = even k, then the
//    NG little-endian uint16 mantissas, zero padding to the row stride).
//
// Exactness.  Every operation is IEEE binary64 with round-to-nearest-even
// through the __d*_rn intrinsics, so nothing is contracted into an FMA; the
// group error is summed in numpy's own order for a contiguous 128-element
// reduction (eight running sums r[j] over elements j, j+8, ..., then
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7))): thread j of a group's eight threads
// owns r[j] and the tree is three xor-shuffles.  The shared exponent
// e = ceil(log2(max s)) + 1 is left to the caller (host libm / numpy), since
// it is a single scalar per matrix.
//
// The input matrix is float32 (w_f64 = 0) or float64 (w_f64 = 1); the
// reference converts either to float64 first, which float32 does exactly.
//
// Work: one group per 8 threads, 32 groups per 256-thread CTA; the search
// costs 17 divisions per weight, so the kernel is FP64-issue bound (a 9B
// checkpoint quantizes in seconds, against hours for the host reference).
#include <cstdint>

#include <cuda_runtime.h>

#include "../../include/f5b200.h"
#include "f5_capi_util.h"

namespace f5 {

constexpr int QG = 128;            // group size of the W4 wire format
constexpr int QPT = QG / 8;        // weights per thread
constexpr int QCTA = 256;          // 32 groups per CTA
constexpr int QALPHA_MAX = 64;

struct QuantScaleArgs {
  const void *w;                   // [N][K] row-major, float or double
  const double *sal;               // [K] per-channel error weights (nullable)
  double *best_s;                  // [N][NG]
  unsigned long long *smax_bits;   // max over best_s (positive: bit order = value order)
  long long ngroups;
  int K, NG, nalpha;
  double alpha[QALPHA_MAX];
};

template <class T>
__global__ void __launch_bounds__(QCTA) k_quant_scale(const QuantScaleArgs a) {
  const long long gi = (long long)blockIdx.x * (QCTA / 8) + (threadIdx.x >> 3);
  const int j = threadIdx.x & 7;
  const bool live = gi < a.ngroups;
  const long long row = live ? gi / a.NG : 0;
  const int grp = live ? (int)(gi % a.NG) : 0;
  const T *src = static_cast<const T *>(a.w) + row * a.K + (long long)grp * QG + j;
  double x[QPT], sw[QPT];
  double amax = 0.0;
#pragma unroll
  for (int i = 0; i < QPT; ++i) {
    x[i] = live ? (double)src[8 * i] : 0.0;
    sw[i] = a.sal ? a.sal[grp * QG + 8 * i + j] : 1.0;
    amax = fmax(amax, fabs(x[i]));
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) amax = fmax(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const double smax = fmax(amax, 1e-12);
  const double s7 = __ddiv_rn(smax, 7.0);
  double best_s = s7, best_e = __longlong_as_double(0x7ff0000000000000ll);   // +inf
  for (int k = 0; k < a.nalpha; ++k) {
    const double s = __dmul_rn(s7, a.alpha[k]);
    double r = 0.0;
#pragma unroll
    for (int i = 0; i < QPT; ++i) {
      double q = rint(__ddiv_rn(x[i], s));
      q = fmin(fmax(q, -8.0), 7.0);
      const double d = __dsub_rn(__dmul_rn(q, s), x[i]);
      double e2 = __dmul_rn(d, d);
      if (a.sal) e2 = __dmul_rn(e2, sw[i]);
      r = i == 0 ? e2 : __dadd_rn(r, e2);
    }
    r = __dadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 1));
    r = __dadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 2));
    r = __dadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 4));
    if (r < best_e) {   // every thread of the group holds the same r
      best_e = r;
      best_s = s;
    }
  }
  if (live && j == 0) {
    a.best_s[gi] = best_s;
    atomicMax(a.smax_bits, (unsigned long long)__double_as_longlong(best_s));
  }
}

struct QuantPackArgs {
  const void *w;         // [N][K], float or double
  const double *best_s;  // [N][NG]
  uint8_t *img;          // [N][stride], zero-filled by the caller
  int8_t *w4;            // [N][K] codes (nullable)
  uint16_t *m_out;       // [N][NG] mantissas (nullable)
  long long ngroups;
  int K, NG, stride;
  double to_m, to_eff;   // 2^(15-e), 2^(e-15)
};

template <class T>
__global__ void __launch_bounds__(QCTA) k_quant_pack(const QuantPackArgs a) {
  const long long gi = (long long)blockIdx.x * (QCTA / 8) + (threadIdx.x >> 3);
  const int j = threadIdx.x & 7;
  if (gi >= a.ngroups) return;   // whole groups leave together: the shuffles below stay within a group
  const long long row = gi / a.NG;
  const int grp = (int)(gi % a.NG);
  double mr = rint(__dmul_rn(a.best_s[gi], a.to_m));
  mr = fmin(fmax(mr, 1.0), 65535.0);
  const uint32_t m = (uint32_t)mr;
  const double eff = __dmul_rn((double)m, a.to_eff);
  const T *src = static_cast<const T *>(a.w) + row * a.K + (long long)grp * QG + j;
  uint8_t *dst = a.img + row * a.stride + (grp * QG + j) / 2;
  const unsigned mask = __activemask();
#pragma unroll
  for (int i = 0; i < QPT; ++i) {
    double q = rint(__ddiv_rn((double)src[8 * i], eff));
    q = fmin(fmax(q, -8.0), 7.0);
    const int c = (int)q;
    if (a.w4) a.w4[row * a.K + grp * QG + 8 * i + j] = (int8_t)c;
    const int hi = __shfl_xor_sync(mask, c, 1);   // odd k of this pair
    if (!(j & 1)) dst[4 * i] = (uint8_t)((c & 0xF) | ((hi & 0xF) << 4));
  }
  if (j == 0) {
    uint8_t *ms = a.img + row * a.stride + a.K / 2 + 2 * grp;
    ms[0] = (uint8_t)(m & 0xFF);
    ms[1] = (uint8_t)(m >> 8);
    if (a.m_out) a.m_out[gi] = (uint16_t)m;
  }
}

}  // namespace f5

using namespace f5;

int f5_quant_w4_scales(const void *d_w, int w_f64, int N, int K, int g, const double *alpha, int nalpha,
                       const double *d_salience, double *d_best_s, uint64_t *d_smax_bits, void *stream) {
  if (!d_w || !d_best_s || !d_smax_bits || N <= 0 || K <= 0)
    return set_error(F5_EINVAL, "f5_quant_w4_scales: bad arguments");
  if (g != QG || K % QG) return set_error(F5_EINVAL, "f5_quant_w4_scales: g must be 128 and divide K=%d", K);
  if (nalpha < 0 || nalpha > QALPHA_MAX || (nalpha > 0 && !alpha))
    return set_error(F5_EINVAL, "f5_quant_w4_scales: nalpha %d outside [0, %d]", nalpha, QALPHA_MAX);
  QuantScaleArgs a = {};
  a.w = d_w;
  a.sal = d_salience;
  a.best_s = d_best_s;
  a.smax_bits = reinterpret_cast<unsigned long long *>(d_smax_bits);
  a.K = K;
  a.NG = K / QG;
  a.ngroups = (long long)N * a.NG;
  a.nalpha = nalpha;
  for (int i = 0; i < nalpha; ++i) a.alpha[i] = alpha[i];
  const long long blocks = (a.ngroups + QCTA / 8 - 1) / (QCTA / 8);
  if (blocks > 0x7fffffffll) return set_error(F5_EINVAL, "f5_quant_w4_scales: matrix too large");
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(d_smax_bits, 0, sizeof(uint64_t), st);
  if (e == cudaSuccess) {
    if (w_f64) k_quant_scale<double><<<(unsigned)blocks, QCTA, 0, st>>>(a);
    else k_quant_scale<float><<<(unsigned)blocks, QCTA, 0, st>>>(a);
    e = cudaGetLastError();
  }
  return cuda_status(e, "f5_quant_w4_scales");
}

int f5_quant_w4_pack(const void *d_w, int w_f64, int N, int K, int g, const double *d_best_s, int e_shared,
                     uint8_t *d_img, int8_t *d_w4, uint16_t *d_m, void *stream) {
  if (!d_w || !d_best_s || !d_img || N <= 0 || K <= 0) return set_error(F5_EINVAL, "f5_quant_w4_pack: bad arguments");
  int st = check_matrix_shape(N, K, g);
  if (st) return st;
  if (g != QG) return set_error(F5_EINVAL, "f5_quant_w4_pack: g must be 128");
  if (e_shared < -1000 || e_shared > 1000) return set_error(F5_EINVAL, "f5_quant_w4_pack: exponent %d", e_shared);
  QuantPackArgs a = {};
  a.w = d_w;
  a.best_s = d_best_s;
  a.img = d_img;
  a.w4 = d_w4;
  a.m_out = d_m;
  a.K = K;
  a.NG = K / QG;
  a.ngroups = (long long)N * a.NG;
  a.stride = row_stride(K, g);
  a.to_m = ldexp(1.0, 15 - e_shared);
  a.to_eff = ldexp(1.0, e_shared - 15);
  const long long blocks = (a.ngroups + QCTA / 8 - 1) / (QCTA / 8);
  if (blocks > 0x7fffffffll) return set_error(F5_EINVAL, "f5_quant_w4_pack: matrix too large");
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(d_img, 0, (size_t)N * a.stride, s);
  if (e == cudaSuccess) {
    if (w_f64) k_quant_pack<double><<<(unsigned)blocks, QCTA, 0, s>>>(a);
    else k_quant_pack<float><<<(unsigned)blocks, QCTA, 0, s>>>(a);
    e = cudaGetLastError();
  }
  return cuda_status(e, "f5_quant_w4_pack");
}
