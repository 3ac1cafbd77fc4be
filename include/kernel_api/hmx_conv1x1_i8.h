/* candidate_kernel of kernels/expert/hmx_conv1x1_i8/kernel_api.h:11
 * 1x1 convolution: out[p][co] = sx12 field of In[p] . W[co] + bias[co]. */
#ifndef HEXCUDA_KAPI_HMX_CONV1X1_I8_H
#define HEXCUDA_KAPI_HMX_CONV1X1_I8_H
#include <stdint.h>
void candidate_kernel(const uint8_t *In, const int8_t *W, const int32_t *bias, int32_t *out, int n);
#endif
