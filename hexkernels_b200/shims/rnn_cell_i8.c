/* candidate_kernel for rnn_cell_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/rnn_cell_i8.h"
void candidate_kernel(const int8_t *Wx, const int8_t *Wh, const int32_t *b, const int8_t *x, const int8_t *h_prev, int8_t *h_t, int H, int I, int32_t mult, int shift, int8_t zp, const int8_t *tanh_lut) {
    hexcuda_host_rnn_cell_i8(Wx, Wh, b, x, h_prev, h_t, H, I, mult, shift, zp, tanh_lut);
}
