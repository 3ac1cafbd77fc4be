/* candidate_kernel for i8_dot_i32_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_dot_i32_dma.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int n, int32_t *out) {
    hexcuda_host_reduce_int(a, b, HEXCUDA_ELEM_I8, n, HEXCUDA_RED_DOT, out);
}
