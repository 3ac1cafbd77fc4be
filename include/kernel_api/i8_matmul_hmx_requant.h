/* candidate_kernel of kernels/expert/i8_matmul_hmx_requant/kernel_api.h:16
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int8 out = low 8 bits. */
#ifndef HEXCUDA_KAPI_I8_MATMUL_HMX_REQUANT_H
#define HEXCUDA_KAPI_I8_MATMUL_HMX_REQUANT_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, int8_t *out, int n);
#endif
