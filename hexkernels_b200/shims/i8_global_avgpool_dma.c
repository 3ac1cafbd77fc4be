/* candidate_kernel for i8_global_avgpool_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_global_avgpool_dma.h"
void candidate_kernel(const int8_t *a, int n, int8_t *out) {
    int32_t r[2];
    if (hexcuda_host_reduce_int(a, NULL, HEXCUDA_ELEM_I8, n, HEXCUDA_RED_MEAN, r)) return;
    out[0] = (int8_t)r[0];
}
