/* candidate_kernel for epilogue_requant_i32_i8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int32_t *acc, int8_t *out, int n, int32_t mult, int shift) {
    oracle_requant_ew(acc, 0, NULL, 0, n, ORACLE_RQ_PRE_A, 0, mult, shift, 0, 0, -128, 127, -128, 127, NULL, out);
}
