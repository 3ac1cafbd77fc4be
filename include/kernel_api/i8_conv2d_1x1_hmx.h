/* candidate_kernel of kernels/expert/i8_conv2d_1x1_hmx/kernel_api.h:17
 * 1x1 convolution out[co][p] = HMX field of W[co] . in[:, p] (uint16). */
#ifndef HEXCUDA_KAPI_I8_CONV2D_1X1_HMX_H
#define HEXCUDA_KAPI_I8_CONV2D_1X1_HMX_H
#include <stdint.h>
/* the task's fixed shape */
#define CONV_CIN 64
#define CONV_COUT 64
#define CONV_P 64
void candidate_kernel(const uint8_t *in, const int8_t *W, uint16_t *out, int n);
#endif
