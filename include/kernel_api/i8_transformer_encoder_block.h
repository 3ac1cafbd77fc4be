/* candidate_kernel of kernels/expert/i8_transformer_encoder_block/kernel_api.h:46
 * int8 encoder block: HMX-field self-attention of X with every key, residual, HMX-field FFN, residual. */
#ifndef HEXCUDA_KAPI_I8_TRANSFORMER_ENCODER_BLOCK_H
#define HEXCUDA_KAPI_I8_TRANSFORMER_ENCODER_BLOCK_H
#include <stdint.h>
void candidate_kernel(const uint8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2, const int32_t *b2, const uint8_t *exp_lut, int8_t *out, int S, int D, int Dff);
#endif
