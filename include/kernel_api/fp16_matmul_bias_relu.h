/* candidate_kernel of kernels/expert/fp16_matmul_bias_relu/kernel_api.h:16
 * n x n x k_dim fp16 GEMM, out = (fp16) relu((fp16) acc + bias[j]). */
#ifndef HEXCUDA_KAPI_FP16_MATMUL_BIAS_RELU_H
#define HEXCUDA_KAPI_FP16_MATMUL_BIAS_RELU_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, const hvx_hf *bias, hvx_hf *out, int n, int k_dim);
#endif
