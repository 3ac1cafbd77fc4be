/* candidate_kernel for rescale_i16_i8_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/rescale_i16_i8_dma.h"
void candidate_kernel(const int16_t *a, int8_t *out, int n) {
    hexcuda_host_affine_ew(a, HEXCUDA_ELEM_I16, out, HEXCUDA_ELEM_I8, n, 0, 3, 0, 4, HEXCUDA_ROUND_HALF_AWAY, 1, 0, -128, 127);
}
