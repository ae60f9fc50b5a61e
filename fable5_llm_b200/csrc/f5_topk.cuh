// TOPK-32 capture (see f5_topk.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/f5b200.h"

namespace f5 {

size_t topk32_ws_bytes(long long n);
// vals: n int32 values in arrival order (index = position); out: device
// result; e_x (nullable, device): copied into out->e_x
cudaError_t launch_topk32(const int32_t *vals, long long n, void *ws, f5_topk32 *out, const int *e_x,
                          cudaStream_t st);
// nb independent arrays: vals + i * vals_bs, out[i], e_x[i * ex_bs]; ws holds
// nb * topk32_ws_bytes(n)
cudaError_t launch_topk32_b(const int32_t *vals, long long n, int nb, long long vals_bs, void *ws, f5_topk32 *out,
                            const int *e_x, int ex_bs, cudaStream_t st);

}  // namespace f5
