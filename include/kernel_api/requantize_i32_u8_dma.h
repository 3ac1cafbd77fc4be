/* candidate_kernel of kernels/expert/requantize_i32_u8_dma/kernel_api.h:13-14:
 * out[i] = sat_u8(round_half_away((int64)a[i] * mult >> shift) + zp). */
#ifndef HEXCUDA_KAPI_REQUANTIZE_I32_U8_DMA_H
#define HEXCUDA_KAPI_REQUANTIZE_I32_U8_DMA_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, uint8_t *out, int n,
                      int32_t mult, int shift, uint8_t zp);
#endif
