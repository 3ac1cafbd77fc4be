/* candidate_kernel for i8_weighted_sum on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_weighted_sum.h"
void candidate_kernel(const int8_t *a, const int8_t *w, int n, int32_t *out) {
    hexcuda_host_reduce_int(a, w, HEXCUDA_ELEM_I8, n, HEXCUDA_RED_DOT, out);
}
