/* candidate_kernel of kernels/expert/fp16_attention_av_hmx/kernel_api.h:
 * out = P[n x k_dim] . V[k_dim x n], fp32 accumulate, fp16 out. */
#ifndef HEXCUDA_KAPI_FP16_ATTENTION_AV_HMX_H
#define HEXCUDA_KAPI_FP16_ATTENTION_AV_HMX_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *P, const hvx_hf *V, hvx_hf *out, int n, int k_dim);
#endif
