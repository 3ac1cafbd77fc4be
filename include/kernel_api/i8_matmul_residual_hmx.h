/* candidate_kernel of kernels/expert/i8_matmul_residual_hmx/kernel_api.h:17
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int32 out, + residual[i][j]. */
#ifndef HEXCUDA_KAPI_I8_MATMUL_RESIDUAL_HMX_H
#define HEXCUDA_KAPI_I8_MATMUL_RESIDUAL_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *C, int32_t *out, int n);
#endif
