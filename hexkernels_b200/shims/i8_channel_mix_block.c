/* candidate_kernel for i8_channel_mix_block on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_channel_mix_block.h"
void candidate_kernel(const int8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2, const int32_t *b2, const int8_t *gelu_lut, int8_t *out, int32_t mult1, int shift1, int32_t mult2, int shift2) {
    hexcuda_host_mix_mlp_i8(X, W1, b1, gelu_lut, W2, b2, out, CMIX_TOKENS, CMIX_CHANNELS, CMIX_D_FF, CMIX_CHANNELS, mult1, shift1, mult2, shift2);
}
