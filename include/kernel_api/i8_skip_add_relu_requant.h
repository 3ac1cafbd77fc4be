/* candidate_kernel of kernels/expert/i8_skip_add_relu_requant/kernel_api.h:13
 * elementwise requant: pre add_relu, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_I8_SKIP_ADD_RELU_REQUANT_H
#define HEXCUDA_KAPI_I8_SKIP_ADD_RELU_REQUANT_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, const int8_t *b, int8_t *out, int n, int32_t mult, int shift, int8_t zp);
#endif
