/* candidate_kernel of kernels/expert/dma_stream_requant_i32_i8/kernel_api.h:18
 * elementwise requant: pre a, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_DMA_STREAM_REQUANT_I32_I8_H
#define HEXCUDA_KAPI_DMA_STREAM_REQUANT_I32_I8_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, int8_t *out, int n, int32_t mult, int shift, int8_t zp);
#endif
