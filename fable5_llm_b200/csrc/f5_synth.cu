// Device-side generator of the seeded synthetic model (bench inputs).
//
// Produces byte-for-byte the same images as fable5_llm_b200/synth.py:
// word(i) = mix64(key + (i+1) * GOLDEN) with the splitmix64 finaliser; the
// per-matrix keys are derived on the host and passed in.  Generating 4 GB of
// weights in HBM avoids a host round trip for the benchmark model.
#include <stdint.h>
#include <cuda_runtime.h>

namespace f5 {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
constexpr uint64_t GOLDEN = 0x9E3779B97F4A7C15ull;

// sign-magnitude nibble -> two's complement code (zero-mean law)
__device__ __forceinline__ uint32_t sym_nibble(uint32_t c) {
  const uint32_t m = c & 7u;
  return ((c & 8u) ? (0u - m) : m) & 0xFu;
}
__device__ __forceinline__ uint64_t sym_word(uint64_t w) {
  uint64_t o = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) o |= (uint64_t)sym_nibble((uint32_t)(w >> (4 * i)) & 0xFu) << (4 * i);
  return o;
}

__global__ void k_synth_w4(uint8_t *img, long long nrows, int K, int g, long long row0,
                           uint64_t key_w, uint64_t key_m, int symmetric) {
  const int wpr = K / 16;            // 8-byte weight words per row
  const int NG = K / g;
  const int stride = (K / 128 + (NG + 31) / 32) * 64;
  const int tail = stride - K / 2 - 2 * NG;
  const long long per_row = wpr + NG + tail;
  const long long total = nrows * per_row;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long r = t / per_row;
    const int j = (int)(t - r * per_row);
    uint8_t *row = img + r * (long long)stride;
    const long long gr = row0 + r;
    if (j < wpr) {
      uint64_t w = mix64(key_w + (uint64_t)(gr * wpr + j + 1) * GOLDEN);
      if (symmetric) w = sym_word(w);
      *reinterpret_cast<uint64_t *>(row + 8 * j) = w;
    } else if (j < wpr + NG) {
      const int gi = j - wpr;
      const uint64_t h = mix64(key_m + (uint64_t)(gr * NG + gi + 1) * GOLDEN);
      const uint16_t m = (uint16_t)(0x2000u | (uint32_t)(h & 0x1FFFu));
      *reinterpret_cast<uint16_t *>(row + K / 2 + 2 * gi) = m;
    } else {
      row[K / 2 + 2 * NG + (j - wpr - NG)] = 0;
    }
  }
}

__global__ void k_synth_emb(int16_t *emb, long long nrows, int H, long long row0, uint64_t key_e) {
  const long long total = nrows * H;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long r = t / H;
    const int i = (int)(t - r * H);
    const uint64_t w = mix64(key_e + (uint64_t)((row0 + r) * (H / 4) + i / 4 + 1) * GOLDEN);
    const int sh = 16 * (i & 3);
    const int b0 = (int)((w >> sh) & 0xFF), b1 = (int)((w >> (sh + 8)) & 0xFF);
    emb[t] = (int16_t)(b0 + b1 - 255);
  }
}

cudaError_t launch_synth_w4(uint8_t *img, long long nrows, int K, int g, long long row0,
                            uint64_t key_w, uint64_t key_m, int symmetric, cudaStream_t st) {
  k_synth_w4<<<148 * 8, 256, 0, st>>>(img, nrows, K, g, row0, key_w, key_m, symmetric);
  return cudaGetLastError();
}

cudaError_t launch_synth_emb(int16_t *emb, long long nrows, int H, long long row0, uint64_t key_e,
                             cudaStream_t st) {
  k_synth_emb<<<148 * 8, 256, 0, st>>>(emb, nrows, H, row0, key_e);
  return cudaGetLastError();
}

}  // namespace f5
