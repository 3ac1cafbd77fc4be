/* candidate_kernel of kernels/expert/hmx_matmul_fp16_relu/kernel_api.h:9
 * fp16 GEMM, out = (fp16) max(acc, 0). */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_FP16_RELU_H
#define HEXCUDA_KAPI_HMX_MATMUL_FP16_RELU_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n);
#endif
