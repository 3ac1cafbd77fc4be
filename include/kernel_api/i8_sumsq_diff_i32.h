/* candidate_kernel of kernels/expert/i8_sumsq_diff_i32/kernel_api.h:7
 * sum of squared int8 differences, int32 accumulator. */
#ifndef HEXCUDA_KAPI_I8_SUMSQ_DIFF_I32_H
#define HEXCUDA_KAPI_I8_SUMSQ_DIFF_I32_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, const int8_t *b, int n, int32_t *out);
#endif
