/* candidate_kernel of kernels/expert/hmx_matmul_i8_requant/kernel_api.h:12
 * n x n u8 x s8 GEMM, out = clamp(sx12((acc * 17 + 8) >> 4), -128, 127). */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_I8_REQUANT_H
#define HEXCUDA_KAPI_HMX_MATMUL_I8_REQUANT_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, int8_t *out, int n);
#endif
