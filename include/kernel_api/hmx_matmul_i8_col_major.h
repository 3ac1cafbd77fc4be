/* candidate_kernel of kernels/expert/hmx_matmul_i8_col_major/kernel_api.h:10
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int32 out, column-major. */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_I8_COL_MAJOR_H
#define HEXCUDA_KAPI_HMX_MATMUL_I8_COL_MAJOR_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, int32_t *out, int n);
#endif
