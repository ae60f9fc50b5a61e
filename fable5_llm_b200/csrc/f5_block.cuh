// Block-level integer reductions shared by the vector kernels.
#pragma once
#include "f5_int.cuh"

namespace f5 {

// Sum over the block (any blockDim multiple of 32, <= 1024).  `red` holds
// >= 32 long longs of shared scratch.  Result valid in every thread.
F5_DEV long long block_sum_ll(long long v, long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  long long t = 0;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

F5_DEV unsigned long long block_sum_ull(unsigned long long v, unsigned long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  unsigned long long t = 0;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

F5_DEV unsigned long long block_max_ull(unsigned long long v, unsigned long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  unsigned long long t = 0;
  for (int i = 0; i < nw; ++i) t = red[i] > t ? red[i] : t;
  return t;
}

F5_DEV long long block_max_ll(long long v, long long *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  long long t = red[0];
  for (int i = 1; i < nw; ++i) t = red[i] > t ? red[i] : t;
  return t;
}

}  // namespace f5
