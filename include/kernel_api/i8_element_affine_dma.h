/* candidate_kernel of kernels/expert/i8_element_affine_dma/kernel_api.h:11
 * int64 a * scale + shift, round half away >> s, int8 saturation. */
#ifndef HEXCUDA_KAPI_I8_ELEMENT_AFFINE_DMA_H
#define HEXCUDA_KAPI_I8_ELEMENT_AFFINE_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int8_t *out, int n, int32_t scale, int32_t shift, int s);
#endif
