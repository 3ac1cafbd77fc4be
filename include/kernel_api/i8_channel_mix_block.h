/* candidate_kernel of kernels/expert/i8_channel_mix_block/kernel_api.h:43
 * int8 channel-mixing MLP (TOKENS 8, CHANNELS 16, D_FF 16; kernel_api.h:39-41). */
#ifndef HEXCUDA_KAPI_I8_CHANNEL_MIX_BLOCK_H
#define HEXCUDA_KAPI_I8_CHANNEL_MIX_BLOCK_H
#include <stdint.h>
#define CMIX_TOKENS 8
#define CMIX_CHANNELS 16
#define CMIX_D_FF 16
void candidate_kernel(const int8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2, const int32_t *b2, const int8_t *gelu_lut, int8_t *out, int32_t mult1, int shift1, int32_t mult2, int shift2);
#endif
