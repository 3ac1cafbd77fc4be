/* candidate_kernel of kernels/expert/dma_double_buffer_reduce_i32/kernel_api.h:11
 * whole-array int32 sum, int64 accumulator. */
#ifndef HEXCUDA_KAPI_DMA_DOUBLE_BUFFER_REDUCE_I32_H
#define HEXCUDA_KAPI_DMA_DOUBLE_BUFFER_REDUCE_I32_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, int n, int64_t *out);
#endif
