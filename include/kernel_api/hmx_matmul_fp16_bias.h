/* candidate_kernel of kernels/expert/hmx_matmul_fp16_bias/kernel_api.h:9
 * fp16 GEMM, out = (fp16)(acc + bias[j]). */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_FP16_BIAS_H
#define HEXCUDA_KAPI_HMX_MATMUL_FP16_BIAS_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, const hvx_hf *bias, hvx_hf *out, int n);
#endif
