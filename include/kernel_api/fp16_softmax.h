/* candidate_kernel of kernels/expert/fp16_softmax/kernel_api.h:15: row
 * softmax of an R x C fp16 matrix, fp32 arithmetic. */
#ifndef HEXCUDA_KAPI_FP16_SOFTMAX_H
#define HEXCUDA_KAPI_FP16_SOFTMAX_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *x, hvx_hf *out, int R, int C);
#endif
