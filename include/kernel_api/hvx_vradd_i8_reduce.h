/* candidate_kernel of kernels/expert/hvx_vradd_i8_reduce/kernel_api.h:14
 * sums of 4 consecutive int8 -> int32, g groups. */
#ifndef HEXCUDA_KAPI_HVX_VRADD_I8_REDUCE_H
#define HEXCUDA_KAPI_HVX_VRADD_I8_REDUCE_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int32_t *out, int g);
#endif
