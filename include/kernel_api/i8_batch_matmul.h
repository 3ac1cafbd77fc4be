/* candidate_kernel of kernels/expert/i8_batch_matmul/kernel_api.h:9
 * 4 independent s8 x s8 GEMMs (the reference's BATCH 4), int32 out. */
#ifndef HEXCUDA_KAPI_I8_BATCH_MATMUL_H
#define HEXCUDA_KAPI_I8_BATCH_MATMUL_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K);
#endif
