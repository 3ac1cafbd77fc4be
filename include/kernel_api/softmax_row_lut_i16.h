/* candidate_kernel of kernels/expert/softmax_row_lut_i16/kernel_api.h:25
 * int16 exp-table row softmax. */
#ifndef HEXCUDA_KAPI_SOFTMAX_ROW_LUT_I16_H
#define HEXCUDA_KAPI_SOFTMAX_ROW_LUT_I16_H
#include <stdint.h>
void candidate_kernel(const int16_t *x, int16_t *out, int R, int C, const uint16_t *exp_lut);
#endif
