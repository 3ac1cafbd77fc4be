/* candidate_kernel of kernels/expert/fp16_matmul_leaky_relu_hmx/kernel_api.h:15
 * fp16 GEMM, out = (fp16) leaky((fp16) acc), slope 0.125. */
#ifndef HEXCUDA_KAPI_FP16_MATMUL_LEAKY_RELU_HMX_H
#define HEXCUDA_KAPI_FP16_MATMUL_LEAKY_RELU_HMX_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n, int k_dim);
#endif
