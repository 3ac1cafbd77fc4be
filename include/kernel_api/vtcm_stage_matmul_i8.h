/* candidate_kernel of kernels/expert/vtcm_stage_matmul_i8/kernel_api.h:20
 * int8 GEMM with a narrow X [K,N], low 32 bits of the exact sums. */
#ifndef HEXCUDA_KAPI_VTCM_STAGE_MATMUL_I8_H
#define HEXCUDA_KAPI_VTCM_STAGE_MATMUL_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *X, int32_t *C, int M, int K, int N);
#endif
