/* candidate_kernel of kernels/expert/fp16_matmul_hmx_deepk/kernel_api.h:17
 * n x n x k_dim fp16 GEMM. */
#ifndef HEXCUDA_KAPI_FP16_MATMUL_HMX_DEEPK_H
#define HEXCUDA_KAPI_FP16_MATMUL_HMX_DEEPK_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n, int k_dim);
#endif
