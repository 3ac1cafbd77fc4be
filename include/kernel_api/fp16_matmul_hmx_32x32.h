/* candidate_kernel of kernels/expert/fp16_matmul_hmx_32x32/kernel_api.h:10
 * n^3 fp16 GEMM, fp32 accumulate, one fp16 rounding. */
#ifndef HEXCUDA_KAPI_FP16_MATMUL_HMX_32X32_H
#define HEXCUDA_KAPI_FP16_MATMUL_HMX_32X32_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n);
#endif
