/* candidate_kernel of kernels/expert/rmsnorm_row_fp16/kernel_api.h:22
 * fp16 RMS norm per row (eps 1e-3), per-column gamma. */
#ifndef HEXCUDA_KAPI_RMSNORM_ROW_FP16_H
#define HEXCUDA_KAPI_RMSNORM_ROW_FP16_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *x, const hvx_hf *gamma, hvx_hf *out, int R, int C);
#endif
