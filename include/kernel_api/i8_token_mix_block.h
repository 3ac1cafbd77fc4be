/* candidate_kernel of kernels/expert/i8_token_mix_block/kernel_api.h:41
 * int8 token-mixing MLP (TOKENS 8, CHANNELS 16, D_MIX 16; kernel_api.h:37-39). */
#ifndef HEXCUDA_KAPI_I8_TOKEN_MIX_BLOCK_H
#define HEXCUDA_KAPI_I8_TOKEN_MIX_BLOCK_H
#include <stdint.h>
#define TMIX_TOKENS 8
#define TMIX_CHANNELS 16
#define TMIX_D_MIX 16
void candidate_kernel(const int8_t *X, const int8_t *W, const int32_t *b, const int8_t *W2, const int32_t *b2, int8_t *out, int32_t mult1, int shift1, int32_t mult2, int shift2);
#endif
