/* candidate_kernel of kernels/expert/online_softmax_step_fp16/kernel_api.h:
 * one online-softmax update of (running_max, running_sum, acc[D]) in place. */
#ifndef HEXCUDA_KAPI_ONLINE_SOFTMAX_STEP_FP16_H
#define HEXCUDA_KAPI_ONLINE_SOFTMAX_STEP_FP16_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *scores, const hvx_hf *V,
                      hvx_hf *running_max, hvx_hf *running_sum, hvx_hf *acc,
                      int BLK, int D);
#endif
