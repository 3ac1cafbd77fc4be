/* candidate_kernel of kernels/expert/hvx_vmin_u8/kernel_api.h:12
 * elementwise unsigned uint8 min. */
#ifndef HEXCUDA_KAPI_HVX_VMIN_U8_H
#define HEXCUDA_KAPI_HVX_VMIN_U8_H
#include <stdint.h>
void candidate_kernel(const uint8_t *a, const uint8_t *b, uint8_t *out, int n);
#endif
