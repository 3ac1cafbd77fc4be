/* candidate_kernel for fp16_softmax on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/fp16_softmax.h"
void candidate_kernel(const hvx_hf *x, hvx_hf *out, int R, int C) {
    hexcuda_host_softmax_f16((const uint16_t *)x, (uint16_t *)out, R, C);
}
