/* candidate_kernel of kernels/expert/ffn_down_i8/kernel_api.h:21
 * int8 GEMM with Bt [N,K] + bias + round-half-away requant, int8 out. */
#ifndef HEXCUDA_KAPI_FFN_DOWN_I8_H
#define HEXCUDA_KAPI_FFN_DOWN_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int8_t *out, int M, int N, int K, int32_t scale_mult, int scale_shift);
#endif
