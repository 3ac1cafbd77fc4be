/* candidate_kernel of kernels/expert/dequant_i8_i16_dma/kernel_api.h:12
 * (x - zp) * scale >> shift (floor), int16 saturation. */
#ifndef HEXCUDA_KAPI_DEQUANT_I8_I16_DMA_H
#define HEXCUDA_KAPI_DEQUANT_I8_I16_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int16_t *out, int n, int8_t zp, int32_t scale, int shift);
#endif
