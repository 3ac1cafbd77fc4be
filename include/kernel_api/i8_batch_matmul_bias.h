/* candidate_kernel of kernels/expert/i8_batch_matmul_bias/kernel_api.h:14
 * 4 independent s8 x s8 GEMMs + per-batch column bias, int32 out. */
#ifndef HEXCUDA_KAPI_I8_BATCH_MATMUL_BIAS_H
#define HEXCUDA_KAPI_I8_BATCH_MATMUL_BIAS_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int32_t *C, int M, int N, int K);
#endif
