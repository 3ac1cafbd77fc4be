/* candidate_kernel for hvx_vmax_i8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int8_t *out, int n) {
    oracle_minmax_ew(a, b, 0, ORACLE_ELEM_I8, 0, out, n);
}
