/* candidate_kernel of kernels/expert/fp16_matmul_residual/kernel_api.h:17
 * n x n x k_dim fp16 GEMM, out = (fp16)((fp16) acc + C[i][j]). */
#ifndef HEXCUDA_KAPI_FP16_MATMUL_RESIDUAL_H
#define HEXCUDA_KAPI_FP16_MATMUL_RESIDUAL_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, const hvx_hf *C, hvx_hf *out, int n, int k_dim);
#endif
