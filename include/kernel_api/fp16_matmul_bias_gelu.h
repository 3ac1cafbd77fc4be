/* candidate_kernel of kernels/expert/fp16_matmul_bias_gelu/kernel_api.h:19
 * n x n x k_dim fp16 GEMM, out = (fp16) gelu((fp16) acc + bias[j]), tanh form. */
#ifndef HEXCUDA_KAPI_FP16_MATMUL_BIAS_GELU_H
#define HEXCUDA_KAPI_FP16_MATMUL_BIAS_GELU_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, const hvx_hf *bias, hvx_hf *out, int n, int k_dim);
#endif
