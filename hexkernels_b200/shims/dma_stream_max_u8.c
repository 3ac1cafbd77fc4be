/* candidate_kernel for dma_stream_max_u8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/dma_stream_max_u8.h"
void candidate_kernel(const uint8_t *a, int n, uint8_t *out) {
    int32_t m;
    if (hexcuda_host_reduce_int(a, NULL, HEXCUDA_ELEM_U8, n, HEXCUDA_RED_MAX, &m) == HEXCUDA_OK)
        out[0] = (uint8_t)m;
}
