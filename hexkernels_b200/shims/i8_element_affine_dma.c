/* candidate_kernel for i8_element_affine_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_element_affine_dma.h"
void candidate_kernel(const int8_t *a, int8_t *out, int n, int32_t scale, int32_t shift, int s) {
    hexcuda_host_affine_ew(a, HEXCUDA_ELEM_I8, out, HEXCUDA_ELEM_I8, n, 0, scale, shift, s, HEXCUDA_ROUND_HALF_AWAY, 0, 0, -128, 127);
}
