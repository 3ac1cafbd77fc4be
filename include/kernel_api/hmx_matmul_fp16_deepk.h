/* candidate_kernel of kernels/expert/hmx_matmul_fp16_deepk/kernel_api.h:10:
 * out[i*n+j] = (fp16) sum_k A[i*k_dim+k] * B[k*n+j] (row-major B). */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_FP16_DEEPK_H
#define HEXCUDA_KAPI_HMX_MATMUL_FP16_DEEPK_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n, int k_dim);
#endif
