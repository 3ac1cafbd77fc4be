/* candidate_kernel of kernels/expert/rmsnorm_gain_fp16/kernel_api.h:24
 * fp16 RMS norm per row (eps 1e-3) times one gain per row. */
#ifndef HEXCUDA_KAPI_RMSNORM_GAIN_FP16_H
#define HEXCUDA_KAPI_RMSNORM_GAIN_FP16_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *x, const hvx_hf *gain, hvx_hf *out, int R, int C);
#endif
