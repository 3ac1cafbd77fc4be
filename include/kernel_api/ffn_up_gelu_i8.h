/* candidate_kernel of kernels/expert/ffn_up_gelu_i8/kernel_api.h:17
 * FFN up-projection: s8 x s8 GEMM (Bt) + bias, saturate, GELU table. */
#ifndef HEXCUDA_KAPI_FFN_UP_GELU_I8_H
#define HEXCUDA_KAPI_FFN_UP_GELU_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, const int8_t *gelu_lut, int8_t *out, int M, int N, int K);
#endif
