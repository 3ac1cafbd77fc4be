/* candidate_kernel of kernels/expert/gelu_ffn_residual/kernel_api.h:29
 * int8 GELU FFN with residual and table layernorm. */
#ifndef HEXCUDA_KAPI_GELU_FFN_RESIDUAL_H
#define HEXCUDA_KAPI_GELU_FFN_RESIDUAL_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, const int8_t *W1, const int32_t *b1, const int8_t *gelu_lut, const int8_t *W2, const int32_t *b2, const int8_t *x_res, const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut, int8_t *out, int M, int K, int V, int D);
#endif
