/* candidate_kernel of kernels/expert/i16_gemm/kernel_api.h:8
 * int16 GEMM, int32 accumulator. */
#ifndef HEXCUDA_KAPI_I16_GEMM_H
#define HEXCUDA_KAPI_I16_GEMM_H
#include <stdint.h>
void candidate_kernel(const int16_t *A, const int16_t *B, int32_t *C, int M, int N, int K);
#endif
