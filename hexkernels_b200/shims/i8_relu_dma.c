/* candidate_kernel for i8_relu_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_relu_dma.h"
void candidate_kernel(const int8_t *x, int8_t *out, int n) {
    hexcuda_host_affine_ew(x, HEXCUDA_ELEM_I8, out, HEXCUDA_ELEM_I8, n, 0, 1, 0, 0, HEXCUDA_ROUND_FLOOR, 1, 0, 0, 127);
}
