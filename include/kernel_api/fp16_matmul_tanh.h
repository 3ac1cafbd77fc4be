/* candidate_kernel of kernels/expert/fp16_matmul_tanh/kernel_api.h:17
 * n x n x k_dim fp16 GEMM, out = (fp16) tanh((fp16) acc). */
#ifndef HEXCUDA_KAPI_FP16_MATMUL_TANH_H
#define HEXCUDA_KAPI_FP16_MATMUL_TANH_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n, int k_dim);
#endif
