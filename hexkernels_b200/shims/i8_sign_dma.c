/* candidate_kernel for i8_sign_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_sign_dma.h"
void candidate_kernel(const int8_t *in, int8_t *out, int n) {
    hexcuda_host_affine_ew(in, HEXCUDA_ELEM_I8, out, HEXCUDA_ELEM_I8, n, 0, 1000, 0, 0, HEXCUDA_ROUND_FLOOR, 1, 0, -1, 1);
}
