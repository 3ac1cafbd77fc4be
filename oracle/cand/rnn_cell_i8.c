/* candidate_kernel for rnn_cell_i8 backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const int8_t *Wx, const int8_t *Wh, const int32_t *b, const int8_t *x, const int8_t *h_prev, int8_t *h_t, int H, int I, int32_t mult, int shift, int8_t zp, const int8_t *tanh_lut) {
    oracle_rnn_cell_i8(Wx, Wh, b, x, h_prev, h_t, H, I, mult, shift, zp, tanh_lut);
}
