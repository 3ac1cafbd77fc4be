/* candidate_kernel of kernels/expert/i8_layernorm_dma/kernel_api.h:31
 * int8 row layernorm with an inverse-variance table. */
#ifndef HEXCUDA_KAPI_I8_LAYERNORM_DMA_H
#define HEXCUDA_KAPI_I8_LAYERNORM_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, int8_t *out, int R, int W, const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut);
#endif
