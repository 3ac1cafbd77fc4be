/* candidate_kernel for softmax_row_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/softmax_row_i8.h"
void candidate_kernel(const int8_t *x, uint8_t *out, int R, int C, const uint8_t *exp_lut, const uint16_t *recip_lut) {
    hexcuda_host_lut_softmax_u8(x, out, R, C, exp_lut, recip_lut);
}
