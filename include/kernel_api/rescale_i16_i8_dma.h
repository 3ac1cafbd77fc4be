/* candidate_kernel of kernels/expert/rescale_i16_i8_dma/kernel_api.h:14
 * int16 x 3, round half away >> 4, int8 saturation. */
#ifndef HEXCUDA_KAPI_RESCALE_I16_I8_DMA_H
#define HEXCUDA_KAPI_RESCALE_I16_I8_DMA_H
#include <stdint.h>
void candidate_kernel(const int16_t *a, int8_t *out, int n);
#endif
