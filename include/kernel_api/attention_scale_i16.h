/* candidate_kernel of kernels/expert/attention_scale_i16/kernel_api.h:34
 * int32 scores requantised to int16. */
#ifndef HEXCUDA_KAPI_ATTENTION_SCALE_I16_H
#define HEXCUDA_KAPI_ATTENTION_SCALE_I16_H
#include <stdint.h>
void candidate_kernel(const int32_t *raw, int16_t *out, int M, int N, int32_t scale_mult, int scale_shift);
#endif
