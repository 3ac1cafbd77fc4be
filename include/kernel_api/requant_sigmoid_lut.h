/* candidate_kernel of kernels/expert/requant_sigmoid_lut/kernel_api.h:15
 * elementwise requant: pre a, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_REQUANT_SIGMOID_LUT_H
#define HEXCUDA_KAPI_REQUANT_SIGMOID_LUT_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, int8_t *out, int n, int32_t mult, int shift, int8_t zp, const int8_t lut[256]);
#endif
