/* candidate_kernel of kernels/expert/fp16_rmsnorm/kernel_api.h: one row of n
 * features, eps 1e-3. */
#ifndef HEXCUDA_KAPI_FP16_RMSNORM_H
#define HEXCUDA_KAPI_FP16_RMSNORM_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *x, const hvx_hf *gamma, hvx_hf *out, int n);
#endif
