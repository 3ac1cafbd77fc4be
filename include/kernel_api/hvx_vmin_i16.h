/* candidate_kernel of kernels/expert/hvx_vmin_i16/kernel_api.h:9
 * elementwise signed int16 min. */
#ifndef HEXCUDA_KAPI_HVX_VMIN_I16_H
#define HEXCUDA_KAPI_HVX_VMIN_I16_H
#include <stdint.h>
void candidate_kernel(const int16_t *a, const int16_t *b, int16_t *out, int n);
#endif
