/* candidate_kernel of kernels/expert/i8_l1norm_dma/kernel_api.h:7
 * L1 norm of int8 (|-128| = 128), int32 accumulator. */
#ifndef HEXCUDA_KAPI_I8_L1NORM_DMA_H
#define HEXCUDA_KAPI_I8_L1NORM_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int n, int32_t *out);
#endif
