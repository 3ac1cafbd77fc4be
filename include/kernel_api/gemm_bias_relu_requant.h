/* candidate_kernel of kernels/expert/gemm_bias_relu_requant/kernel_api.h:14
 * s8 GEMM, + bias, ReLU, requant to int8. */
#ifndef HEXCUDA_KAPI_GEMM_BIAS_RELU_REQUANT_H
#define HEXCUDA_KAPI_GEMM_BIAS_RELU_REQUANT_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int8_t *out, int M, int N, int K, int32_t mult, int shift, int8_t zp);
#endif
