// f5_matvec_y32_host_noalloc: the host-buffer matvec without any device
// allocation.
//
// Who needs it: callers that must not call cudaMalloc -- a host whose device
// memory is owned entirely by another allocator (a framework's caching pool
// or a fixed arena that has already reserved the GPU's memory, so a
// cudaMalloc beside it fails or fragments that pool), and latency-critical
// loops that cannot take the device-wide synchronisation cudaMalloc /
// cudaFree imply.  f5_matvec_y32_host allocates and frees its device buffers
// on every call; this variant stages the image, x8, y32, p and the error word
// in one fixed array that the library reserves in device memory, so a call
// only copies and launches.
//
// Contract:
//   - the array is F5_NOALLOC_SCRATCH_BYTES (16 MiB); every GPU that loads
//     the library holds it until the process exits;
//   - a request whose staged size (image + x8 + y32 + p + error word, each
//     256-byte aligned) exceeds it is rejected with F5_EINVAL;
//   - the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, once per device, with that device current); make
//     that first call before any stream capture starts;
//   - every call shares the one array and it keeps the previous call's
//     contents: the error word is cleared on each call, and calls that
//     overlap on the GPU (for instance from two host threads) race;
//   - calls are synchronous on the legacy default stream.
#include <cstddef>
#include <mutex>

#include "../../include/f5b200.h"
#include "f5_capi_util.h"
#include "f5_kernels.cuh"

namespace {

static __device__ __align__(256) unsigned char f5_noalloc_scratch[F5_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char *g_scratch[kMaxDevices] = {};

// device address of the array on the current device (host code cannot use
// the symbol itself: in host code its name is only a host-side stand-in)
int scratch_on_current_device(unsigned char **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return f5::cuda_status(e, "f5_matvec_y32_host_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return f5::set_error(F5_EINVAL, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, f5_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return f5::cuda_status(e == cudaSuccess ? cudaErrorInvalidSymbol : e,
                             "f5_matvec_y32_host_noalloc: cudaGetSymbolAddress");
    g_scratch[dev] = static_cast<unsigned char *>(p);
  }
  *out = g_scratch[dev];
  return F5_OK;
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace

extern "C" int f5_matvec_y32_host_noalloc(const uint8_t *img, int N, int K, int g, int sh, const int8_t *x8,
                                          int32_t *y32, int64_t *p) {
  using namespace f5;
  if (!img || !x8 || !y32) return set_error(F5_EINVAL, "f5_matvec_y32_host_noalloc: null pointer");
  int rc = check_matrix_shape(N, K, g);
  if (rc) return rc;
  const size_t stride = (size_t)row_stride(K, g);
  const size_t off_x8 = align256(stride * (size_t)N);
  const size_t off_y = align256(off_x8 + (size_t)K);
  const size_t off_p = align256(off_y + 4 * (size_t)N);
  const size_t off_err = align256(off_p + (p ? 8 * (size_t)N : 0));
  const size_t total = off_err + 256;
  if (total > F5_NOALLOC_SCRATCH_BYTES)
    return set_error(F5_EINVAL,
                     "f5_matvec_y32_host_noalloc: N=%d K=%d needs %zu bytes of staging, above the %u-byte "
                     "fixed scratch (use f5_matvec_y32_host)",
                     N, K, total, (unsigned)F5_NOALLOC_SCRATCH_BYTES);
  unsigned char *base = nullptr;
  if ((rc = scratch_on_current_device(&base))) return rc;
  uint8_t *d_img = base;
  int8_t *d_x8 = reinterpret_cast<int8_t *>(base + off_x8);
  int32_t *d_y = reinterpret_cast<int32_t *>(base + off_y);
  int64_t *d_p = p ? reinterpret_cast<int64_t *>(base + off_p) : nullptr;
  uint32_t *d_err = reinterpret_cast<uint32_t *>(base + off_err);
  uint32_t herr = 0;
  cudaError_t e;
  if ((e = cudaMemcpy(d_img, img, stride * N, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(d_x8, x8, K, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemset(d_err, 0, sizeof(uint32_t))) != cudaSuccess)
    return cuda_status(e, "f5_matvec_y32_host_noalloc: staging");
  f5_gemv_seg s = {};
  s.w = d_img;
  s.out = d_y;
  s.p_out = d_p;
  s.rows = N;
  s.mode = F5_GM_Y32;
  if ((rc = f5_gemv_dev(&s, 1, K, g, sh, d_x8, nullptr, nullptr, d_err, 0, 0, nullptr))) return rc;
  if ((e = cudaMemcpy(y32, d_y, sizeof(int32_t) * N, cudaMemcpyDeviceToHost)) != cudaSuccess ||
      (p && (e = cudaMemcpy(p, d_p, sizeof(int64_t) * N, cudaMemcpyDeviceToHost)) != cudaSuccess) ||
      (e = cudaMemcpy(&herr, d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_status(e, "f5_matvec_y32_host_noalloc: results");
  if (herr & DERR_Y32_OVERFLOW)
    return set_error(F5_EOVERFLOW, "y32 overflow -- sh miscomputed (ref/w4a8_ref.py:288)");
  if (herr & DERR_TIMEOUT) return set_error(F5_ETIMEOUT, "a bounded device wait gave up");
  return F5_OK;
}
