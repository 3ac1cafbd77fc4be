/* candidate_kernel for i8_min_scalar_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_min_scalar_dma.h"
void candidate_kernel(const int8_t *in, int8_t *out, int n, int8_t c) {
    hexcuda_host_minmax_ew(in, NULL, c, HEXCUDA_ELEM_I8, 1, out, n);
}
