/* candidate_kernel for online_softmax_step_fp16 on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/online_softmax_step_fp16.h"
void candidate_kernel(const hvx_hf *scores, const hvx_hf *V, hvx_hf *running_max,
                      hvx_hf *running_sum, hvx_hf *acc, int BLK, int D) {
    hexcuda_host_online_softmax_step_f16((const uint16_t *)scores, (const uint16_t *)V,
                                         (uint16_t *)running_max, (uint16_t *)running_sum,
                                         (uint16_t *)acc, BLK, D);
}
