/* candidate_kernel of kernels/expert/i8_weighted_sum/kernel_api.h:7
 * int8 weighted sum (dot product), int32 accumulator. */
#ifndef HEXCUDA_KAPI_I8_WEIGHTED_SUM_H
#define HEXCUDA_KAPI_I8_WEIGHTED_SUM_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, const int8_t *w, int n, int32_t *out);
#endif
