/* candidate_kernel for i8_argmin_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_argmin_dma.h"
void candidate_kernel(const int8_t *a, int n, int32_t *out) {
    hexcuda_host_reduce_int(a, NULL, HEXCUDA_ELEM_I8, n, HEXCUDA_RED_ARGMIN, out);
}
