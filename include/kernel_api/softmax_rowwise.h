/* candidate_kernel of kernels/expert/softmax_rowwise/kernel_api.h:20
 * int8 exp-table row softmax, u8 out. */
#ifndef HEXCUDA_KAPI_SOFTMAX_ROWWISE_H
#define HEXCUDA_KAPI_SOFTMAX_ROWWISE_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, uint8_t *out, int R, int C, const uint8_t *exp_lut);
#endif
