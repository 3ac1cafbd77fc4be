/* candidate_kernel of kernels/expert/hvx_vmax_i8/kernel_api.h:9
 * elementwise signed int8 max. */
#ifndef HEXCUDA_KAPI_HVX_VMAX_I8_H
#define HEXCUDA_KAPI_HVX_VMAX_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, const int8_t *b, int8_t *out, int n);
#endif
