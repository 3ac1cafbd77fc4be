/* candidate_kernel of kernels/expert/hmx_conv1x1_fp16/kernel_api.h:10
 * 1x1 convolution = GEMM with W stored [co][ci]. */
#ifndef HEXCUDA_KAPI_HMX_CONV1X1_FP16_H
#define HEXCUDA_KAPI_HMX_CONV1X1_FP16_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *In, const hvx_hf *W, hvx_hf *out, int n);
#endif
