/* candidate_kernel of kernels/expert/hmx_matmul_i8_deepk/kernel_api.h:13
 * A [n,K] u8, B [K,n] s8, out int32 [n,n] = sx12((acc * 17 + 8) >> 4). */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_I8_DEEPK_H
#define HEXCUDA_KAPI_HMX_MATMUL_I8_DEEPK_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, int32_t *out, int n, int K);
#endif
