/* candidate_kernel of kernels/expert/i8_add_bias_sat_dma/kernel_api.h:8
 * x + bias with int8 saturation. */
#ifndef HEXCUDA_KAPI_I8_ADD_BIAS_SAT_DMA_H
#define HEXCUDA_KAPI_I8_ADD_BIAS_SAT_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, int8_t *out, int n, int32_t bias);
#endif
