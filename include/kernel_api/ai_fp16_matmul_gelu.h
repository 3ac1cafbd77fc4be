/* candidate_kernel of kernels/expert/ai_fp16_matmul_gelu/kernel_api.h:8
 * n^3 fp16 GEMM, out = (fp16) gelu((fp16) acc), tanh form. */
#ifndef HEXCUDA_KAPI_AI_FP16_MATMUL_GELU_H
#define HEXCUDA_KAPI_AI_FP16_MATMUL_GELU_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n);
#endif
