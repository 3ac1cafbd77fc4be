/* candidate_kernel of kernels/expert/i8_pointwise_conv_hmx/kernel_api.h:16
 * pointwise convolution out[co][p] = HMX field of W[co] . in[:, p] (uint16). */
#ifndef HEXCUDA_KAPI_I8_POINTWISE_CONV_HMX_H
#define HEXCUDA_KAPI_I8_POINTWISE_CONV_HMX_H
#include <stdint.h>
/* the task's fixed shape */
#define CONV_CIN 96
#define CONV_COUT 64
#define CONV_P 64
void candidate_kernel(const uint8_t *in, const int8_t *W, uint16_t *out, int n);
#endif
