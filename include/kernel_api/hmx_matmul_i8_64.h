/* candidate_kernel of kernels/expert/hmx_matmul_i8_64/kernel_api.h:12
 * n x n u8 x s8 GEMM, out int32 = sx12((acc * 17 + 8) >> 4). */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_I8_64_H
#define HEXCUDA_KAPI_HMX_MATMUL_I8_64_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, int32_t *out, int n);
#endif
