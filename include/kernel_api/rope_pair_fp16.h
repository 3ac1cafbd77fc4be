/* candidate_kernel of kernels/expert/rope_pair_fp16/kernel_api.h:21
 * fp16 rotary embedding of interleaved pairs. */
#ifndef HEXCUDA_KAPI_ROPE_PAIR_FP16_H
#define HEXCUDA_KAPI_ROPE_PAIR_FP16_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *x, const hvx_hf *cos, const hvx_hf *sin, hvx_hf *out, int n_pairs);
#endif
