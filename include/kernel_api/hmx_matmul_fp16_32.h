/* candidate_kernel of kernels/expert/hmx_matmul_fp16_32/kernel_api.h:9
 * n^3 fp16 GEMM. */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_FP16_32_H
#define HEXCUDA_KAPI_HMX_MATMUL_FP16_32_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n);
#endif
