/* candidate_kernel for i8_token_mix_block on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_token_mix_block.h"
void candidate_kernel(const int8_t *X, const int8_t *W, const int32_t *b, const int8_t *W2, const int32_t *b2, int8_t *out, int32_t mult1, int shift1, int32_t mult2, int shift2) {
    hexcuda_host_token_mix_i8(X, W, b, W2, b2, out, TMIX_TOKENS, TMIX_CHANNELS, TMIX_D_MIX, mult1, shift1, mult2, shift2);
}
