/* candidate_kernel of kernels/expert/vtcm_reduce_i32/kernel_api.h:8
 * whole-array int32 sum, int32 out (wraps). */
#ifndef HEXCUDA_KAPI_VTCM_REDUCE_I32_H
#define HEXCUDA_KAPI_VTCM_REDUCE_I32_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, int n, int32_t *out);
#endif
