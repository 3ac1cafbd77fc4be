/* candidate_kernel of kernels/expert/i8_clip_requant_dma/kernel_api.h:15
 * elementwise requant: pre a, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_I8_CLIP_REQUANT_DMA_H
#define HEXCUDA_KAPI_I8_CLIP_REQUANT_DMA_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, int8_t *out, int n, int32_t mult, int shift, int8_t zp, int8_t lo, int8_t hi);
#endif
