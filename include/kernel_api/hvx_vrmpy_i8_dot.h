/* candidate_kernel of kernels/expert/hvx_vrmpy_i8_dot/kernel_api.h:12
 * 4-wide int8 dot products, int32 out. */
#ifndef HEXCUDA_KAPI_HVX_VRMPY_I8_DOT_H
#define HEXCUDA_KAPI_HVX_VRMPY_I8_DOT_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, const int8_t *b, int32_t *out, int g);
#endif
