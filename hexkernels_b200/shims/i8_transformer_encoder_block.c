/* candidate_kernel for i8_transformer_encoder_block on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_transformer_encoder_block.h"
void candidate_kernel(const uint8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2, const int32_t *b2, const uint8_t *exp_lut, int8_t *out, int S, int D, int Dff) {
    hexcuda_host_encoder_block_i8(X, W1, b1, W2, b2, exp_lut, out, S, D, Dff);
}
