/* candidate_kernel of kernels/expert/i8_matmul_hmx_64x64/kernel_api.h:14
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); uint16 out = unsigned 12-bit field. */
#ifndef HEXCUDA_KAPI_I8_MATMUL_HMX_64X64_H
#define HEXCUDA_KAPI_I8_MATMUL_HMX_64X64_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, uint16_t *out, int n);
#endif
