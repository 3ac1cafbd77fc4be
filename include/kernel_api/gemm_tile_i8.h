/* candidate_kernel of kernels/expert/gemm_tile_i8/kernel_api.h:11
 * s8 x s8 GEMM, B given as Bt [N,K], int32 out. */
#ifndef HEXCUDA_KAPI_GEMM_TILE_I8_H
#define HEXCUDA_KAPI_GEMM_TILE_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K);
#endif
