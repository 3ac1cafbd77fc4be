/* candidate_kernel for softmax_rowwise on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/softmax_rowwise.h"
void candidate_kernel(const int8_t *x, uint8_t *out, int R, int C, const uint8_t *exp_lut) {
    hexcuda_host_lut_softmax_u8(x, out, R, C, exp_lut, NULL);
}
