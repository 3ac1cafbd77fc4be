/* candidate_kernel of kernels/expert/fp16_attention_qkt_hmx/kernel_api.h:20:
 * out[i*n+j] = (fp16) sum_d Q[i*k_dim+d] * K[j*k_dim+d] (fp32 accumulate):
 * the column-major-B fp16 GEMM, also the M=N=K=8192 benchmark case. */
#ifndef HEXCUDA_KAPI_FP16_ATTENTION_QKT_HMX_H
#define HEXCUDA_KAPI_FP16_ATTENTION_QKT_HMX_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, hvx_hf *out, int n, int k_dim);
#endif
