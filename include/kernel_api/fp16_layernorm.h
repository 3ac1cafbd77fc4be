/* candidate_kernel of kernels/expert/fp16_layernorm/kernel_api.h:17-18: one
 * row of n features, eps 1e-3. */
#ifndef HEXCUDA_KAPI_FP16_LAYERNORM_H
#define HEXCUDA_KAPI_FP16_LAYERNORM_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *x, const hvx_hf *gamma, const hvx_hf *beta,
                      hvx_hf *out, int n);
#endif
