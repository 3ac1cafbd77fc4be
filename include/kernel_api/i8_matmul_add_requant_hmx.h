/* candidate_kernel of kernels/expert/i8_matmul_add_requant_hmx/kernel_api.h:16
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int8 saturated out, + residual[i][j]. */
#ifndef HEXCUDA_KAPI_I8_MATMUL_ADD_REQUANT_HMX_H
#define HEXCUDA_KAPI_I8_MATMUL_ADD_REQUANT_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, const int8_t *residual, int8_t *out, int n);
#endif
