/* candidate_kernel for dma_double_buffer_reduce_i32 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int32_t *a, int n, int64_t *out) {
    oracle_reduce_int(a, NULL, ORACLE_ELEM_I32, n, ORACLE_RED_SUM64, out);
}
