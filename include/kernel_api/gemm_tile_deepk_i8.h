/* candidate_kernel of kernels/expert/gemm_tile_deepk_i8/kernel_api.h:17
 * s8 x s8 GEMM, B row-major [K,N], int32 out (deep K). */
#ifndef HEXCUDA_KAPI_GEMM_TILE_DEEPK_I8_H
#define HEXCUDA_KAPI_GEMM_TILE_DEEPK_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K);
#endif
