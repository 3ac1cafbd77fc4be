/* candidate_kernel for softmax_row_lut_i16 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/softmax_row_lut_i16.h"
void candidate_kernel(const int16_t *x, int16_t *out, int R, int C, const uint16_t *exp_lut) {
    hexcuda_host_lut_softmax_i16(x, out, R, C, exp_lut);
}
