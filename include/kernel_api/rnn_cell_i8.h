/* candidate_kernel of kernels/expert/rnn_cell_i8/kernel_api.h:30
 * one int8 RNN step with a tanh table. */
#ifndef HEXCUDA_KAPI_RNN_CELL_I8_H
#define HEXCUDA_KAPI_RNN_CELL_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *Wx, const int8_t *Wh, const int32_t *b, const int8_t *x, const int8_t *h_prev, int8_t *h_t, int H, int I, int32_t mult, int shift, int8_t zp, const int8_t *tanh_lut);
#endif
