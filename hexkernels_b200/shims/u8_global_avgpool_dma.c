/* candidate_kernel for u8_global_avgpool_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/u8_global_avgpool_dma.h"
void candidate_kernel(const uint8_t *a, int n, uint8_t *out) {
    int32_t r[2];
    if (hexcuda_host_reduce_int(a, NULL, HEXCUDA_ELEM_U8, n, HEXCUDA_RED_MEAN, r)) return;
    out[0] = (uint8_t)r[0];
}
