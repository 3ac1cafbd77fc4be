/* candidate_kernel for i8_element_affine_dma backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const int8_t *a, int8_t *out, int n, int32_t scale, int32_t shift, int s) {
    oracle_affine_ew(a, ORACLE_ELEM_I8, out, ORACLE_ELEM_I8, n, 0, scale, shift, s, 0, 0, 0, -128, 127);
}
