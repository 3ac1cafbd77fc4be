/* candidate_kernel of kernels/expert/softmax_row_i8/kernel_api.h:32
 * int8 exp-table row softmax normalised by a reciprocal table. */
#ifndef HEXCUDA_KAPI_SOFTMAX_ROW_I8_H
#define HEXCUDA_KAPI_SOFTMAX_ROW_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, uint8_t *out, int R, int C, const uint8_t *exp_lut, const uint16_t *recip_lut);
#endif
