/* candidate_kernel for i8_add_bias_sat_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_add_bias_sat_dma.h"
void candidate_kernel(const int8_t *x, int8_t *out, int n, int32_t bias) {
    hexcuda_host_affine_ew(x, HEXCUDA_ELEM_I8, out, HEXCUDA_ELEM_I8, n, 0, 1, bias, 0, HEXCUDA_ROUND_FLOOR, 1, 0, -128, 127);
}
