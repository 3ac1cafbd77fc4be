/* candidate_kernel of kernels/expert/i8_sumsq_i32/kernel_api.h:5
 * sum of squares of int8, int32 accumulator. */
#ifndef HEXCUDA_KAPI_I8_SUMSQ_I32_H
#define HEXCUDA_KAPI_I8_SUMSQ_I32_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int n, int32_t *out);
#endif
