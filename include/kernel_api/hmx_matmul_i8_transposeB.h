/* candidate_kernel of kernels/expert/hmx_matmul_i8_transposeB/kernel_api.h:11
 * acc = sum_k A[i][k] * Bt[j][k], out int32 = sx12((acc * 17 + 8) >> 4). */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_I8_TRANSPOSEB_H
#define HEXCUDA_KAPI_HMX_MATMUL_I8_TRANSPOSEB_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *Bt, int32_t *out, int n);
#endif
