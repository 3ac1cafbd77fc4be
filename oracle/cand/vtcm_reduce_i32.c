/* candidate_kernel for vtcm_reduce_i32 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int32_t *a, int n, int32_t *out) {
    oracle_reduce_int(a, NULL, ORACLE_ELEM_I32, n, ORACLE_RED_SUM, out);
}
