// Shared helpers of the C ABI translation units.
#pragma once
#include <cuda_runtime.h>

namespace f5 {
int set_error(int status, const char *fmt, ...);
int cuda_status(cudaError_t e, const char *where);
int sm_count();
int check_matrix_shape(int N, int K, int g);
int row_stride(int K, int g);
}  // namespace f5
