/* candidate_kernel for hvx_vmax_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/hvx_vmax_i8.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int8_t *out, int n) {
    hexcuda_host_minmax_ew(a, b, 0, HEXCUDA_ELEM_I8, 0, out, n);
}
